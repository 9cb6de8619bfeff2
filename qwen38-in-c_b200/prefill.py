"""Long prefill through the projection set (benchmark configuration 4) -- a
harness over libq35cuda's C-ABI, shared by bench.py and the GPU tests.

The engine's batch prefill (qwen35-c/src/q35_model.c:980-1104) runs every
projection of a layer on all M tokens at once through q35_mm_fp8_batch
(q35_deltanet.c:387-390, q35_attn.c:305-307, q35_model.c:972-975).  One
layer here issues the same projections, in the same order, on the weights of
a ``stack.Stack`` (this rank's tensor-parallel shards):

  DeltaNet: qkv, z = GEMM(x)           column-parallel
            o = GEMM_out(z)             row-parallel (the caller-batched out)
  GQA:      q, k, v = GEMM(x)           column-parallel
            o = GEMM_o(attn)            row-parallel (attn: the local heads'
                                        attention output, a stand-in)
  MLP:      gate, up = GEMM(o)          column-parallel
            y = GEMM_down(gate)         row-parallel

Every GEMM is the tcgen05 kernel with one caller workspace, through
``q35cu_gemm_fp8_multi``: the projections that read the same input (qkv | z,
q | k | v, gate | up) as one preparation and one launch over their row
blocks together; on the fp32 outputs of earlier projections it rounds them
to bf16 as it prepares them (no separate conversion pass).  The recurrence, attention and swiglu arithmetic between
projections is not part of the matmul path and is not run.

Tensor parallelism (world > 1): "literal" all-gathers each column-parallel
output ([M, N/p] fp32 per rank) and all-reduces each row-parallel partial
([M, 5120] fp32) with NCCL; "paired" (Megatron) drops the all-gathers -- the
row-parallel projection consumes the local shard.  Under TP the tokens are
cut into `slabs` row slabs (a slab's rows are contiguous in every [M, N]
buffer): each projection runs slab by slab on the compute stream, and each
slab's collective runs on a second stream as soon as that slab's GEMM is
done, so the exchange of slab i overlaps the GEMMs of slab i + 1 onwards;
a GEMM that consumes an all-reduced output (gate/up after out/o) waits for
that slab's all-reduce only.
"""
from __future__ import annotations

import q35cu
import stack


class PrefillLayers:
    """Device buffers for M tokens through one layer of each kind of `st`."""

    def __init__(self, st: "stack.Stack", m: int = 8192, scheme: str = "literal", seed: int = 4321,
                 slabs: int | None = None):
        import torch

        assert scheme in ("literal", "paired")
        self.st, self.m, self.scheme = st, m, scheme
        self.world = st.world
        self.slabs = (4 if st.world > 1 else 1) if slabs is None else slabs
        assert m % self.slabs == 0
        self.comm = torch.cuda.Stream(device=st.dev) if st.world > 1 else None
        # Under TP the collectives run beside the GEMMs, which are persistent
        # (one CTA per SM): a GEMM CTA whose SM a collective holds starts late
        # and holds up its tiles.  The literal scheme, whose all-gathers keep
        # NCCL busy through most of a layer, leaves NCCL 32 SMs; the paired
        # scheme's two all-reduces per layer cost less than reserved SMs of
        # GEMM.  Measured at TP 2, M = 8192, e4m3 GEMM, ms per pass: literal
        # 337 / 341 / 300 / 314 with 0 / 16 / 32 / 48 reserved, paired 256 /
        # 259 with 0 / 16.  Q35_PREFILL_RESERVE_SMS overrides.
        default = "32" if scheme == "literal" else "0"
        self.reserve = int(__import__("os").environ.get("Q35_PREFILL_RESERVE_SMS", default)) if st.world > 1 else 0
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

    def layer_reserved(self, L, stream=None, keep=None) -> None:
        """layer() with this scheme's SM reservation in force for its GEMMs."""
        lib = q35cu.load()
        q35cu.check(lib.q35cu_gemm_reserve_sms(self.reserve))
        try:
            self.layer(L, stream, keep)
        finally:
            q35cu.check(lib.q35cu_gemm_reserve_sms(0))

    def layer(self, L, stream=None, keep=None) -> None:
        """Issue one layer's projections (asynchronous on `stream`, the
        current stream if None; the collectives of a TP run go on the
        second stream, joined back before this returns).  `keep`, a dict,
        receives clones of every GEMM's bf16 input (for checks)."""
        import torch

        literal = self.scheme == "literal" and self.world > 1
        cs = stream if stream is not None else torch.cuda.current_stream(self.st.dev)
        S = self.slabs
        ms = self.m // S
        rows = [slice(i * ms, (i + 1) * ms) for i in range(S)]
        if self.comm is not None:
            self.comm.wait_stream(cs)  # buffers written before this layer

        def gemm(ws, xin, youts, names, waits=None):
            """the GEMMs of weights ws on one input, slab by slab on cs (slab
            i after waits[i], if given): one q35cu_gemm_fp8_multi call per
            slab over all of ws (one preparation, one launch).  An fp32 input
            is rounded to bf16 inside that preparation, with no separate
            conversion pass.  Returns the event after each slab."""
            f32 = xin.dtype == torch.float32
            if keep is not None:
                kx = xin.to(torch.bfloat16) if f32 else xin.clone()
                for n in names:
                    keep[n] = kx
            evs = []
            for i, r in enumerate(rows):
                if waits is not None:
                    cs.wait_event(waits[i])
                # one workspace: slabs in order on cs
                q35cu.gemm_multi(ws, xin[r], [y[r] for y in youts], self.work, cs)
                if self.comm is not None:
                    ev = torch.cuda.Event()
                    ev.record(cs)
                    evs.append(ev)
            return evs

        def exchange(evs, buf, out=None):
            """each slab's all-gather (out given) or all-reduce on the second
            stream, after that slab's GEMM; the events after each"""
            done = []
            per = buf.numel() // S
            for i, r in enumerate(rows):
                self.comm.wait_event(evs[i])
                if out is not None:
                    q35cu.allgather(buf[r], out[i * per * self.world:(i + 1) * per * self.world], self.comm)
                else:
                    q35cu.allreduce(buf[r], self.comm)
                ev = torch.cuda.Event()
                ev.record(self.comm)
                done.append(ev)
            return done

        # the column-parallel projections of x (qkv | z, q | k | v) as one GEMM
        evs = gemm([p.w for p in L.col_in], self.x, [self.col[p.name] for p in L.col_in],
                   [p.name for p in L.col_in])
        if literal:
            for p in L.col_in:
                exchange(evs, self.col[p.name], self.gath[p.name])
        src = self.col["z"] if L.kind == "dn" else self.attn
        evs = gemm([L.attn_out.w], src, [self.o], [L.attn_out.name])
        # under TP, the gate | up GEMM's slab i waits for that slab's all-reduce only
        done = exchange(evs, self.o) if self.world > 1 else None
        g_evs = gemm([L.gate.w, L.up.w], self.o, [self.gu["gate"], self.gu["up"]], ["gate", "up"], done)
        if literal:
            exchange(g_evs, self.gu["gate"], self.gu_g["gate"])
            exchange(g_evs, self.gu["up"], self.gu_g["up"])
        evs = gemm([L.down.w], self.gu["gate"], [self.y], [L.down.name])
        if self.world > 1:
            exchange(evs, self.y)
            cs.wait_stream(self.comm)

    def flops(self, L) -> float:
        """This rank's GEMM flops for one layer of L's kind."""
        return 2.0 * self.m * sum(p.window[1] * p.window[3] for p in L.col_in + [L.attn_out, L.gate, L.up, L.down])
