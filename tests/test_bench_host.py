"""bench.py's host-side logic on CPU: the CPU description, the CPU stream the
reference arm times, and the child-process isolation of the extras (a failing
extra yields {"error": ...} instead of taking the headline line with it)."""
from __future__ import annotations

import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import bench  # noqa: E402


def test_cpu_info_counts_the_allowed_cpus():
    info = bench.cpu_info()
    assert info["logical_cpus"] == len(os.sched_getaffinity(0))
    assert info["physical_cores"] is None or 1 <= info["physical_cores"] <= info["logical_cpus"]
    assert info["model"]


def test_cpu_stream_layers_are_distinct_rotations(orc):
    """Layers other than 0 and 3 hold byte-rotated copies of the seeded
    weights of their kind: distinct memory, the same bytes."""
    cs = bench.CpuStream(n_layers=4)
    kinds = [k for k, _ in cs.layers]
    assert kinds == ["dn", "dn", "dn", "gqa"]
    W0, s0 = cs.layers[0][1]["gate"]
    W1, s1 = cs.layers[1][1]["gate"]
    assert W0.shape == W1.shape and not np.shares_memory(W0, W1)
    assert not np.array_equal(W0, W1)
    assert np.array_equal(np.bincount(W0.ravel(), minlength=256), np.bincount(W1.ravel(), minlength=256))
    # the seeded layer matches the generator the GPU stack uses
    import stack

    Wg, sg = orc.synth_fp8(stack.seed_of(0, "gate"), stack.MLP, stack.HIDDEN)
    assert np.array_equal(Wg, W0) and np.array_equal(sg, s0)
    outs = []
    cs.step(lambda W, s, x: outs.append(orc.mm_fp8(W, s, x)) or outs[-1],
            lambda Ws, Ss, x: [orc.mm_fp8(w, s, x) for w, s in zip(Ws, Ss)])
    assert len(outs) == 8 and all(np.isfinite(o).all() for o in outs)


def test_failing_extra_reports_an_error():
    """No GPU here: the configuration-0 child fails, and run_child turns that
    into an error entry instead of raising."""
    args = bench.parse(["--gpus", "1"])
    r = bench.run_child("c0", args, timeout=600)
    assert isinstance(r, dict) and "error" in r and r["error"].startswith("rc=")
