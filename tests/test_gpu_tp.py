"""Tensor parallelism on real GPUs: one process per GPU, NCCL through libq35cuda.

Needs at least two GPUs (skipped otherwise).  Each rank

* checks q35cu_allreduce_f32 / q35cu_allgather_f32 on integer-valued data
  (exact in fp32);
* generates its shard window of each projection in HBM
  (q35cu_weight_synth_fp8 with the window of q35cu_shard_window), runs the
  decode GEMV on it and combines the ranks the way the decode step does:
  all-gather for column-parallel (must equal the unsharded GPU product
  bit for bit: every row is computed whole), all-reduce for row-parallel
  (the K sum is split across ranks; must meet the guarded 1e-5 GEMV bound
  against the CPU oracle);
* checks the one-shot NVLink collectives (q35cu_p2p_*): exact on integer
  data, bit-identical to NCCL (at two ranks a sum has one order), correct
  across CUDA-graph replays (their sequence numbers live on the device);
* runs two layers of the decode-step harness with both schemes on the three
  collective backends (NCCL, the one-shot peer-memory kernels, and the
  exchange fused into the GEMV epilogue, q35cu_multi_fp8_tp) and checks that
  the replicated outputs agree bit for bit across ranks and between the
  backends, and that the fused all-gather fills the same gathered buffers;
* runs the same step as one decode chain (q35cu_chain_*, a cooperative launch
  with the exchanges fused) and checks it equals the fused step bit for bit.

The shard layout and combination rules follow the reference's projections
(qwen35-c/src/q35_model.c: q/k/v/z/gate/up produce rows, o/out/down reduce
over K); the reference itself is single-process.
"""
from __future__ import annotations

import json
import os
import socket

import pytest

SHAPES = [  # (rows, cols, mode) with mode 0 = column-parallel, 1 = row-parallel
    (17408, 5120, 0),   # gate / up
    (10240, 5120, 0),   # qkv
    (1024, 5120, 0),    # k / v
    (5120, 17408, 1),   # down
    (5120, 6144, 1),    # out / o
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen38-in-c_b200"), os.path.join(repo, "oracle"), here):
        sys.path.insert(0, p)
    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle
    import q35cu
    import stack
    from parity import gemv_report

    torch.cuda.set_device(rank)
    q35cu.check(q35cu.load().q35cu_set_device(rank))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    uid = [q35cu.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    q35cu.tp_init(rank, world, uid[0])
    rep = {"rank": rank}

    # collectives on integer-valued data
    n = 4099
    buf = torch.arange(n, dtype=torch.float32, device="cuda") * (rank + 1)
    q35cu.allreduce(buf)
    send = torch.full((777,), float(rank), device="cuda")
    recv = torch.empty(777 * world, device="cuda")
    q35cu.allgather(send, recv)
    torch.cuda.synchronize()
    rep["allreduce_exact"] = bool(torch.equal(buf.cpu(), torch.arange(n, dtype=torch.float32) * (world * (world + 1) // 2)))
    rep["allgather_exact"] = bool(torch.equal(recv.cpu(), torch.arange(world, dtype=torch.float32).repeat_interleave(777)))

    # one-shot NVLink collectives: exact on integer data, bit-identical to NCCL
    # (at two ranks a sum has one order), stable across CUDA-graph replays
    hs = [None] * world
    dist.all_gather_object(hs, q35cu.p2p_handle())
    q35cu.p2p_open(rank, world, hs)
    buf = torch.arange(n, dtype=torch.float32, device="cuda") * (rank + 1)
    q35cu.p2p_allreduce(buf)
    recv.zero_()
    q35cu.p2p_allgather(send, recv)
    torch.cuda.synchronize()
    rep["p2p_allreduce_exact"] = bool(torch.equal(buf.cpu(), torch.arange(n, dtype=torch.float32) * (world * (world + 1) // 2)))
    rep["p2p_allgather_exact"] = bool(torch.equal(recv.cpu(), torch.arange(world, dtype=torch.float32).repeat_interleave(777)))
    v = torch.randn(5120, generator=torch.Generator().manual_seed(100 + rank)).cuda()
    a_nccl, a_p2p = v.clone(), torch.empty_like(v)
    q35cu.allreduce(a_nccl)
    q35cu.p2p_allreduce(v, a_p2p)
    torch.cuda.synchronize()
    rep["p2p_equals_nccl"] = bool(torch.equal(a_nccl.cpu(), a_p2p.cpu()))
    src = torch.empty(5120, device="cuda")
    dst = torch.empty(5120, device="cuda")
    s_ = torch.cuda.Stream()
    s_.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s_):
        with torch.cuda.graph(g, stream=s_):
            q35cu.p2p_allreduce(src, dst, stream=s_)
    torch.cuda.current_stream().wait_stream(s_)
    ok = True
    for it in range(5):
        src.copy_(torch.full((5120,), float(it * 10 + rank)))
        g.replay()
        torch.cuda.synchronize()
        ok &= bool(torch.equal(dst.cpu(), torch.full((5120,), float(world * it * 10 + world * (world - 1) // 2))))
    del g
    rep["p2p_graph_replays"] = ok

    # sharded projections against the whole weight
    orc = oracle.Oracle()
    rep["shapes"] = []
    for rows, cols, mode in SHAPES:
        seed = 77 + rows * 3 + cols
        x = torch.randn(cols, generator=torch.Generator().manual_seed(cols)).to(torch.float32)
        xd = x.cuda()
        r0, nr, c0, nc = q35cu.shard_window(rows, cols, mode, rank, world)
        w = q35cu.Weight.synth_fp8(seed, rows, cols, window=(r0, nr, c0, nc))
        if mode == 0:
            y_loc = torch.empty(nr, device="cuda")
            q35cu.gemv(w, xd, y_loc)
            y_tp = torch.empty(nr * world, device="cuda")
            q35cu.allgather(y_loc, y_tp)
        else:
            y_tp = torch.empty(rows, device="cuda")
            q35cu.gemv(w, xd[c0:c0 + nc].contiguous(), y_tp)
            q35cu.allreduce(y_tp)
        torch.cuda.synchronize()
        w.free()
        if rank == 0:
            full = q35cu.Weight.synth_fp8(seed, rows, cols)
            y_full = torch.empty(rows, device="cuda")
            q35cu.gemv(full, xd, y_full)
            torch.cuda.synchronize()
            entry = {"rows": rows, "cols": cols, "mode": mode}
            if mode == 0:
                entry["bit_exact"] = bool(torch.equal(y_tp.cpu()[:rows], y_full.cpu()))
            else:
                Wf, scf = full.download_fp8()
                y64, a = orc.mm_fp8_f64(Wf, scf, x.numpy())
                y_ref = orc.mm_fp8(Wf, scf, x.numpy())
                r = gemv_report(y_tp.cpu().numpy(), y_ref, y64, a)
                entry["ok"] = r["ok"]
                entry["max_guarded_rel"] = r["max_guarded_rel"]
            full.free()
            rep["shapes"].append(entry)

    # two layers of the decode step, both schemes, both collective backends:
    # replicated outputs agree across ranks, and P2P equals NCCL (two ranks)
    st = stack.Stack(rank, world, n_layers=2, scheme="literal")
    st.x.copy_(torch.randn(st.x.shape, generator=torch.Generator().manual_seed(5)).cuda())
    outs = {}
    for coll in ("nccl", "p2p", "fused"):
        st.coll = coll
        for scheme in ("literal", "paired"):
            st.scheme = scheme
            st.step()
            torch.cuda.synchronize()
            y = st.y.clone()
            ys = [torch.empty_like(y).cpu() for _ in range(world)]
            dist.all_gather_object(ys, y.cpu())
            rep[f"stack_{coll}_{scheme}_finite"] = bool(torch.isfinite(y).all())
            rep[f"stack_{coll}_{scheme}_replicated"] = all(torch.equal(ys[0], t) for t in ys)
            outs[(coll, scheme)] = y.cpu()
    rep["stack_p2p_equals_nccl"] = all(torch.equal(outs[("nccl", sc)], outs[("p2p", sc)]) for sc in ("literal", "paired"))
    rep["stack_fused_equals_p2p"] = all(torch.equal(outs[("fused", sc)], outs[("p2p", sc)]) for sc in ("literal", "paired"))
    # the fused all-gather fills the same gathered buffers as the collective
    st.coll, st.scheme = "p2p", "literal"
    st.step()
    g_p2p = (st.col_full.clone(), st.gu_full.clone())
    st.coll = "fused"
    st.col_full.zero_()
    st.gu_full.zero_()
    st.step()
    torch.cuda.synchronize()
    rep["fused_gather_equals_p2p"] = bool(torch.equal(g_p2p[0], st.col_full) and torch.equal(g_p2p[1], st.gu_full))
    # the decode chain (one cooperative launch per step, exchanges fused)
    # equals the fused per-projection step, both schemes, twice in a row
    for scheme in ("literal", "paired"):
        st.coll, st.scheme = "fused", scheme
        st.step()
        torch.cuda.synchronize()
        ref = st.y.clone()
        ok = True
        for _ in range(2):
            st.y.fill_(float("nan"))
            st.step_chain()
            torch.cuda.synchronize()
            ok &= bool(torch.equal(ref, st.y))
        rep[f"chain_{scheme}_equals_fused"] = ok
    st.free()
    status = q35cu.C.c_uint32(0)
    q35cu.check(q35cu.load().q35cu_device_status(q35cu.C.byref(status), 1))
    rep["device_status"] = int(status.value)
    dist.barrier()
    q35cu.p2p_close()
    q35cu.tp_finalize()
    with open(os.path.join(out_dir, f"tp_gpu_rank{rank}.json"), "w") as f:
        json.dump(rep, f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_tp_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp

    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (found {torch.cuda.device_count()})")
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    reps = [json.loads((tmp_path / f"tp_gpu_rank{r}.json").read_text()) for r in range(world)]
    for rep in reps:
        assert rep["allreduce_exact"] and rep["allgather_exact"], rep
        assert rep["p2p_allreduce_exact"] and rep["p2p_allgather_exact"], rep
        assert rep["p2p_equals_nccl"] and rep["p2p_graph_replays"], rep
        assert rep["device_status"] == 0, rep
        for coll in ("nccl", "p2p", "fused"):
            for scheme in ("literal", "paired"):
                key = f"stack_{coll}_{scheme}"
                assert rep[key + "_finite"] and rep[key + "_replicated"], (key, rep)
        assert rep["stack_p2p_equals_nccl"], rep
        assert rep["stack_fused_equals_p2p"] and rep["fused_gather_equals_p2p"], rep
        assert rep["chain_literal_equals_fused"] and rep["chain_paired_equals_fused"], rep
    shapes = reps[0]["shapes"]
    assert len(shapes) == len(SHAPES)
    for e in shapes:
        if e["mode"] == 0:
            assert e["bit_exact"], e
        else:
            assert e["ok"], e
