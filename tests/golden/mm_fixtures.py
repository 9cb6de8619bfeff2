"""Regenerate qwen35-c's matmul known-answer fixtures (tests/fixtures/mm).

The reference's fixture generator (qwen35-c/tools/gen_matmul_fixture.py:8-52)
draws every case from one numpy ``default_rng(7)`` stream, in manifest
order: weights ``N(0,1)*0.5`` cast to e4m3fn (or ``*0.25`` to bf16), a
``U[0.5,1)`` block-scale grid cast to bf16, then ``x ~ N(0,1)``.  The
expected output is the float64 product of the f32 dequantised weights with
x.  Because the draws must replay the same stream to reproduce the bytes,
the draw order here is necessarily the reference's; the code is this
project's own.

Two of the reference's blobs are not in the mounted snapshot
(``qkvlike_fp8.w8``, ``deep_bf16.w16``).  Replaying the stream recreates
them; their neighbours ``.x/.sc/.yref`` -- which are present and pinned in
``ref_sha256.json`` -- prove the replay is exact.

Usage:  python tests/golden/mm_fixtures.py OUTDIR   (writes the 8 cases)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

CASES = [  # name, rows, cols, fp8   (qwen35-c/tools/gen_matmul_fixture.py:45-52)
    ("tiny_fp8", 3, 5, True),
    ("edge_fp8", 129, 129, True),
    ("exact1_fp8", 128, 128, True),
    ("wide_fp8", 16, 5120, True),
    ("deep_fp8", 5120, 16, True),
    ("qkvlike_fp8", 10240, 5120, True),
    ("mid_bf16", 256, 128, False),
    ("deep_bf16", 2048, 5120, False),
]
TOL = 5e-4  # qwen35-c/tools/gen_matmul_fixture.py:43, checked as tol + tol*|yref|
HERE = os.path.dirname(os.path.abspath(__file__))
PINS = os.path.join(HERE, "ref_sha256.json")


def generate() -> dict:
    """Return {case: {ext: bytes}} for every case, replaying seed 7."""
    import ml_dtypes

    f8, bf = ml_dtypes.float8_e4m3fn, ml_dtypes.bfloat16
    rng = np.random.default_rng(7)
    out = {}
    for name, rows, cols, fp8 in CASES:
        files = {}
        if fp8:
            w = (rng.standard_normal((rows, cols)).astype(np.float32) * 0.5).astype(f8)
            br, bc = (rows + 127) // 128, (cols + 127) // 128
            s = (rng.random((br, bc)).astype(np.float32) * 0.5 + 0.5).astype(bf)
            x = rng.standard_normal(cols).astype(np.float32)
            s32 = s.astype(np.float32)
            s_full = np.repeat(np.repeat(s32, 128, axis=0)[:rows], 128, axis=1)[:, :cols]
            sw = w.astype(np.float32) * s_full                 # f32, exact products
            yref = sw.astype(np.float64) @ x.astype(np.float64)
            files["w8"] = w.view(np.uint8).tobytes()
            files["sc"] = s.view(np.uint16).tobytes()
        else:
            w = (rng.standard_normal((rows, cols)).astype(np.float32) * 0.25).astype(bf)
            x = rng.standard_normal(cols).astype(np.float32)
            yref = w.astype(np.float64) @ x.astype(np.float64)
            files["w16"] = w.view(np.uint16).tobytes()
        files["x"] = x.tobytes()
        files["yref"] = yref.astype(np.float64).tobytes()
        out[name] = files
    return out


def load_case(files: dict, name: str):
    """Typed arrays for one case: (W, sc or None, x, yref)."""
    _, rows, cols, fp8 = next(c for c in CASES if c[0] == name)
    x = np.frombuffer(files["x"], np.float32).copy()
    yref = np.frombuffer(files["yref"], np.float64).copy()
    if fp8:
        W = np.frombuffer(files["w8"], np.uint8).reshape(rows, cols).copy()
        sc = np.frombuffer(files["sc"], np.uint16).reshape((rows + 127) // 128, (cols + 127) // 128).copy()
        return W, sc, x, yref
    W = np.frombuffer(files["w16"], np.uint16).reshape(rows, cols).copy()
    return W, None, x, yref


def sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def pins() -> dict:
    with open(PINS) as f:
        return json.load(f)


def yref_f32_digest(yref_bytes: bytes) -> str:
    """sha256 of the expected output rounded to fp32.

    The fp64 ``yref`` depends on the BLAS summation order in its last bit
    (2 of 10240 qkvlike entries differ by one fp64 ulp between machines);
    rounded to fp32 it does not, so this digest pins the product itself.
    """
    return sha256(np.frombuffer(yref_bytes, np.float64).astype(np.float32).tobytes())


def pin_from_reference(fixture_dir: str) -> tuple[dict, dict]:
    """sha256 of every fixture file the reference ships, and of each yref
    rounded to fp32 (run where the reference tree exists)."""
    pinned, yref32 = {}, {}
    for name, *_ in CASES:
        for ext in ("w8", "sc", "w16", "x", "yref"):
            p = os.path.join(fixture_dir, f"{name}.{ext}")
            if os.path.exists(p):
                with open(p, "rb") as f:
                    b = f.read()
                pinned[f"{name}.{ext}"] = sha256(b)
                if ext == "yref":
                    yref32[name] = yref_f32_digest(b)
    return pinned, yref32


if __name__ == "__main__":
    if len(sys.argv) >= 2 and sys.argv[1] == "--pin":
        if len(sys.argv) > 2:
            src = sys.argv[2]
        elif os.environ.get("Q35_REF"):  # the reference's qwen35-c directory
            src = os.path.join(os.environ["Q35_REF"], "tests", "fixtures", "mm")
        else:
            sys.exit("usage: mm_fixtures.py --pin FIXTURE_DIR (or set Q35_REF to the qwen35-c tree)")
        files, yref32 = pin_from_reference(src)
        data = {"source": "qwen35-c/tests/fixtures/mm", "files": files, "yref_f32": yref32,
                "fnv1a_reference_outputs": {
                    # printed by the reference test_mm (AVX2 and scalar builds agree)
                    "tiny_fp8": "ed487374cb551695", "edge_fp8": "cdcd943179b1af31",
                    "exact1_fp8": "d11a5a7cb593bd3f", "wide_fp8": "a3f64f5366e12f6f",
                    "deep_fp8": "e4c3a13ff2ad13a0"}}
        with open(PINS, "w") as f:
            json.dump(data, f, indent=1, sort_keys=True)
        print(f"pinned {len(data['files'])} files -> {PINS}")
        sys.exit(0)
    outdir = sys.argv[1]
    os.makedirs(outdir, exist_ok=True)
    for name, files in generate().items():
        for ext, b in files.items():
            with open(os.path.join(outdir, f"{name}.{ext}"), "wb") as f:
                f.write(b)
    print(f"wrote {len(CASES)} cases to {outdir}")
