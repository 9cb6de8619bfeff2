"""Tensor-parallel host logic on CPU: world-size-2 gloo ranks (spawned).

Each rank takes its shard window from libq35cuda's q35cu_shard_window (host
only), generates that window of the global synthetic weight, multiplies it
with the CPU oracle and combines the ranks' results the way the GPU path
does (all-gather for column-parallel, all-reduce for row-parallel).  The
combined result must equal the unsharded product: bit-for-bit for
column-parallel (each row is computed whole), within the guarded 1e-5 rule
for row-parallel (the K sum is split across ranks).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

SHAPES = [  # (rows, cols) of the projections, as in the decode stack
    (17408, 5120),   # gate / up (column)
    (10240, 5120),   # qkv (column)
    (1024, 5120),    # k / v (column)
    (5120, 17408),   # down (row)
    (5120, 6144),    # out / o (row)
    (300, 520),      # ragged edge blocks
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen38-in-c_b200"), os.path.join(repo, "oracle"), here):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import oracle
    import q35cu
    from parity import gemv_report

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    orc = oracle.Oracle()
    report = []
    for rows, cols in SHAPES:
        x = orc.synth_act(11, (cols,))
        # column-parallel: split output rows, all-gather
        r0, nr, c0, nc = q35cu.shard_window(rows, cols, q35cu.SHARD_COLUMN, rank, world)
        W, sc = orc.synth_fp8(rows * 3 + cols, rows, cols, row0=r0, col0=c0, nrows=nr, ncols=nc)
        y_local = torch.from_numpy(orc.mm_fp8(W, sc, x))
        sizes = [None] * world
        dist.all_gather_object(sizes, nr)
        parts = [torch.empty(n) for n in sizes]
        dist.all_gather(parts, y_local) if len(set(sizes)) == 1 else [
            dist.broadcast(parts[r] if r != rank else y_local, src=r) for r in range(world)]
        if len(set(sizes)) != 1:
            parts[rank] = y_local
        y_col = torch.cat(parts).numpy()
        # row-parallel: split the K range, x sliced, all-reduce the partial sums
        r0, nr, c0, nc = q35cu.shard_window(rows, cols, q35cu.SHARD_ROW, rank, world)
        W, sc = orc.synth_fp8(rows * 3 + cols, rows, cols, row0=r0, col0=c0, nrows=nr, ncols=nc)
        y_part = torch.from_numpy(orc.mm_fp8(W, sc, np.ascontiguousarray(x[c0:c0 + nc])))
        dist.all_reduce(y_part)
        y_row = y_part.numpy()
        if rank == 0:
            Wf, scf = orc.synth_fp8(rows * 3 + cols, rows, cols)
            y_full = orc.mm_fp8(Wf, scf, x)
            y64, a = orc.mm_fp8_f64(Wf, scf, x)
            rep = gemv_report(y_row, y_full, y64, a)
            report.append((rows, cols, bool(np.array_equal(y_col.view(np.uint32), y_full.view(np.uint32))),
                           rep["ok"], rep["max_guarded_rel"]))
    if rank == 0:
        with open(os.path.join(out_dir, "tp_report.txt"), "w") as f:
            for r in report:
                f.write(" ".join(str(v) for v in r) + "\n")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_sharding_gloo(tmp_path, world):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    lines = (tmp_path / "tp_report.txt").read_text().split("\n")
    rows = [ln.split() for ln in lines if ln.strip()]
    assert len(rows) == len(SHAPES)
    for rws, cls, col_exact, row_ok, rel in rows:
        assert col_exact == "True", (rws, cls)
        assert row_ok == "True", (rws, cls, rel)
