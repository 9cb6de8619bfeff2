"""The 64-layer FP8 decode weight stream (benchmark configuration 3), on
1..8 GPUs with tensor parallelism -- a harness over libq35cuda's C-ABI.

Layer pattern and projection shapes follow the reference model
(qwen35-c/src/q35_model.c:877-959 decode step; shapes from its config,
.wayfinder/research/qwen3.8-config.json): 64 layers, every 4th a GQA layer
(48 Gated-DeltaNet + 16 GQA), hidden 5120, MLP 17408.

One decode step chains the projections of every layer for one token, the
way the engine's forward_one calls the matmul (q35_deltanet.c:329,360,
q35_attn.c:273-275,262, q35_model.c:934,937):

  DeltaNet: [qkv 10240 | z 6144] = multi(x_l)      (q35_mm_fp8_multi4)
            o   = out(z)              5120x6144     (q35_mm_fp8)
  GQA:      [q 12288 | k 1024 | v 1024] = multi(x_l)
            o   = o_proj(q[:6144])    5120x6144
  MLP:      [gate 17408 | up 17408] = multi(o)
            y_l = down(gate)          5120x17408

x_l is a fresh N(0,1) [5120] vector per layer (the configuration's input);
the attention / recurrence / swiglu arithmetic between projections is not
part of the matmul path and is not run (the chain feeds each projection the
previous projection's output of the right length instead).

Tensor parallelism over `world` ranks (one process per GPU):
  column-parallel (qkv, z, q, k, v, gate, up): rank r holds a 128-aligned
      block of output rows; its output shard is all-gathered (NCCL) in the
      "literal" scheme, or used in place in the "paired" scheme (the
      following row-parallel projection consumes exactly the local shard);
  row-parallel (out, o, down): rank r holds the matching block of input
      columns and consumes the K-slice of its input; the partial outputs
      are all-reduced (NCCL sum).
Every rank generates its own shards of the same global matrices with the
seeded generator, so results do not depend on the world size.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import q35cu

HIDDEN = 5120
MLP = 17408
N_LAYERS = 64
GQA_EVERY = 4  # layer i is GQA when i % 4 == 3 (3:1 pattern)

DN_COL = [("qkv", 10240), ("z", 6144)]
GQA_COL = [("q", 12288), ("k", 1024), ("v", 1024)]
OUT_K = 6144  # out / o projection input width


def layer_kinds(n_layers: int = N_LAYERS):
    return ["gqa" if i % GQA_EVERY == GQA_EVERY - 1 else "dn" for i in range(n_layers)]


def projection_shapes(n_layers: int = N_LAYERS):
    """[(layer, name, rows, cols, kind)] for the whole stack, kind col/row."""
    out = []
    for i, kind in enumerate(layer_kinds(n_layers)):
        for name, rows in (DN_COL if kind == "dn" else GQA_COL):
            out.append((i, name, rows, HIDDEN, "col"))
        out.append((i, "out" if kind == "dn" else "o", HIDDEN, OUT_K, "row"))
        out.append((i, "gate", MLP, HIDDEN, "col"))
        out.append((i, "up", MLP, HIDDEN, "col"))
        out.append((i, "down", HIDDEN, MLP, "row"))
    return out


def weight_bytes(n_layers: int = N_LAYERS) -> int:
    return sum(r * c for _, _, r, c, _ in projection_shapes(n_layers))


def scale_bytes(n_layers: int = N_LAYERS) -> int:
    return sum(4 * ((r + 127) // 128) * ((c + 127) // 128) for _, _, r, c, _ in projection_shapes(n_layers))


def seed_of(layer: int, name: str, base: int = 0x5EED) -> int:
    return (base * 1000003 + layer * 131 + sum(ord(c) * 7 ** i for i, c in enumerate(name))) & 0xFFFFFFFFFFFF


@dataclass
class Proj:
    name: str
    rows: int          # global
    cols: int          # global
    kind: str          # "col" or "row"
    w: q35cu.Weight    # this rank's shard
    window: tuple      # (row0, nrows, col0, ncols)


@dataclass
class Layer:
    kind: str
    col_in: list = field(default_factory=list)   # the multi projections fed by x_l
    attn_out: Proj | None = None
    gate: Proj | None = None
    up: Proj | None = None
    down: Proj | None = None


class Stack:
    """Device-resident weights + activations for one rank; ``step()`` issues
    one decode step on a stream (capturable in a CUDA graph)."""

    def __init__(self, rank: int = 0, world: int = 1, n_layers: int = N_LAYERS, scheme: str = "literal",
                 seed: int = 0x5EED, device=None, coll: str = "nccl"):
        import torch

        assert scheme in ("literal", "paired")
        assert coll in ("nccl", "p2p", "fused")
        self.rank, self.world, self.scheme, self.n_layers = rank, world, scheme, n_layers
        # collectives between projections: NCCL, the one-shot NVLink
        # peer-memory kernels of libq35cuda (q35cu_p2p_*, opened by the
        # caller), or "fused": the same exchange inside the GEMVs' epilogues
        # (q35cu_multi_fp8_tp) with no collective kernel at all
        self.coll = coll
        self.dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.layers: list[Layer] = []
        self.weights: list[q35cu.Weight] = []
        self.local_weight_bytes = 0
        for i, kind in enumerate(layer_kinds(n_layers)):
            L = Layer(kind)
            for name, rows in (DN_COL if kind == "dn" else GQA_COL):
                L.col_in.append(self._proj(i, name, rows, HIDDEN, "col", seed))
            L.attn_out = self._proj(i, "out" if kind == "dn" else "o", HIDDEN, OUT_K, "row", seed)
            L.gate = self._proj(i, "gate", MLP, HIDDEN, "col", seed)
            L.up = self._proj(i, "up", MLP, HIDDEN, "col", seed)
            L.down = self._proj(i, "down", HIDDEN, MLP, "row", seed)
            self.layers.append(L)
        f32 = dict(dtype=torch.float32, device=self.dev)
        self.x = torch.empty((n_layers, HIDDEN), **f32)        # per-layer inputs
        self.y = torch.empty((n_layers, HIDDEN), **f32)        # per-layer outputs
        # column outputs: local shard buffers and, for the literal scheme, gathered buffers
        maxcol = max(sum(p.window[1] for p in L.col_in) for L in self.layers)
        self.col_local = torch.empty((maxcol,), **f32)
        self.col_full = torch.empty((maxcol * world,), **f32)
        gu = self.layers[0].gate.window[1]
        self.gu_local = torch.empty((2 * gu,), **f32)
        self.gu_full = torch.empty((2 * gu * world,), **f32)
        self.o_buf = torch.empty((HIDDEN,), **f32)
        self.kernels_per_step = None

    def _proj(self, layer, name, rows, cols, kind, seed) -> Proj:
        mode = q35cu.SHARD_COLUMN if kind == "col" else q35cu.SHARD_ROW
        win = q35cu.shard_window(rows, cols, mode, self.rank, self.world)
        w = q35cu.Weight.synth_fp8(seed_of(layer, name, seed), rows, cols, window=win)
        self.weights.append(w)
        self.local_weight_bytes += win[1] * win[3]
        return Proj(name, rows, cols, kind, w, win)

    # -- one decode step ---------------------------------------------------
    def step(self, stream=None) -> None:
        """Issue the whole 64-layer step on `stream` (torch current stream if None)."""
        literal = self.scheme == "literal" and self.world > 1
        for i, L in enumerate(self.layers):
            xi = self.x[i]
            # column-parallel projections fed by x_l, outputs packed [p0 | p1 | ...]
            outs, off = [], 0
            for p in L.col_in:
                n = p.window[1]
                outs.append(self.col_local[off:off + n])
                off += n
            fused = self.coll == "fused" and self.world > 1
            if fused and literal:
                q35cu.multi_tp([p.w for p in L.col_in], xi, outs, q35cu.TP_ALLGATHER, self.col_full, stream)
            else:
                q35cu.multi([p.w for p in L.col_in], xi, outs, 1, stream)
                if literal:
                    self._allgather(self.col_local[:off], self.col_full[:off * self.world], stream)
            # out / o consume this rank's K-slice of their input: for DeltaNet the
            # local z shard IS z[c0:c0+nc] (same 128-aligned split of 6144); for
            # GQA the first nc values of the local q shard stand in for the
            # attention output of the local heads (world 1: q[:6144])
            ao = L.attn_out
            nc = ao.window[3]
            src = outs[-1] if L.kind == "dn" else outs[0]
            if fused:
                q35cu.gemv_tp(ao.w, src[:nc], self.o_buf, q35cu.TP_ALLREDUCE, None, stream)
            else:
                q35cu.gemv(ao.w, src[:nc], self.o_buf, 1, stream)
                if self.world > 1:
                    self._allreduce(self.o_buf, stream)
            # MLP: gate/up column-parallel, down row-parallel on the gate shard
            g_n = L.gate.window[1]
            gu = [self.gu_local[:g_n], self.gu_local[g_n:2 * g_n]]
            if fused and literal:
                q35cu.multi_tp([L.gate.w, L.up.w], self.o_buf, gu, q35cu.TP_ALLGATHER, self.gu_full, stream)
            else:
                q35cu.multi([L.gate.w, L.up.w], self.o_buf, gu, 1, stream)
                if literal:
                    self._allgather(self.gu_local[:2 * g_n], self.gu_full[:2 * g_n * self.world], stream)
            if fused:
                q35cu.gemv_tp(L.down.w, self.gu_local[:g_n], self.y[i], q35cu.TP_ALLREDUCE, None, stream)
            else:
                q35cu.gemv(L.down.w, self.gu_local[:g_n], self.y[i], 1, stream)
                if self.world > 1:
                    self._allreduce(self.y[i], stream)

    # -- the same step as one decode chain (q35cu_chain_*) -------------------
    def build_chain(self, scheme: str | None = None):
        """A q35cu.Chain with the ops of step() (TP exchanges fused into the
        GEMV epilogues when world > 1)."""
        scheme = scheme or self.scheme
        literal = scheme == "literal" and self.world > 1
        tp = self.world > 1
        ch = q35cu.Chain()
        for i, L in enumerate(self.layers):
            outs, off = [], 0
            for p in L.col_in:
                n = p.window[1]
                outs.append(self.col_local[off:off + n])
                off += n
            ch.add([p.w for p in L.col_in], self.x[i], outs,
                   q35cu.TP_ALLGATHER if literal else 0, self.col_full if literal else None)
            ao = L.attn_out
            src = outs[-1] if L.kind == "dn" else outs[0]
            ch.add([ao.w], src[:ao.window[3]], [self.o_buf], q35cu.TP_ALLREDUCE if tp else 0)
            g_n = L.gate.window[1]
            gu = [self.gu_local[:g_n], self.gu_local[g_n:2 * g_n]]
            ch.add([L.gate.w, L.up.w], self.o_buf, gu,
                   q35cu.TP_ALLGATHER if literal else 0, self.gu_full if literal else None)
            ch.add([L.down.w], self.gu_local[:g_n], [self.y[i]], q35cu.TP_ALLREDUCE if tp else 0)
        return ch

    def step_chain(self, stream=None) -> None:
        """step() as one cooperative launch (the chain is built on first use)."""
        if not hasattr(self, "_chains"):
            self._chains = {}
        ch = self._chains.get(self.scheme)
        if ch is None:
            ch = self._chains[self.scheme] = self.build_chain(self.scheme)
        ch.run(stream)

    def _allreduce(self, buf, stream) -> None:
        if self.coll == "p2p":
            q35cu.p2p_allreduce(buf, stream=stream)
        else:
            q35cu.allreduce(buf, stream)

    def _allgather(self, send, recv, stream) -> None:
        if self.coll == "p2p":
            q35cu.p2p_allgather(send, recv, stream)
        else:
            q35cu.allgather(send, recv, stream)

    def launches_per_step(self) -> int:
        """Kernels (this library's) + collectives one step issues on this rank."""
        per_layer_k = 4  # multi, out/o, multi(gate,up), down
        per_layer_c = 0 if self.world == 1 else (4 if self.scheme == "literal" else 2)
        return self.n_layers * per_layer_k, self.n_layers * per_layer_c

    def free(self) -> None:
        for ch in getattr(self, "_chains", {}).values():
            ch.free()
        self._chains = {}
        for w in self.weights:
            w.free()
        self.weights = []
