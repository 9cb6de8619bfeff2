"""The safetensors preload (q35cu_preload_safetensors through libq35plat's
q35_plat_mmap_prefetch): the engine maps its shards and binds matmul
operands as pointers into the mappings (qwen35-c/src/q35_model.c:204-208,
252-273), then prefetches every shard (q35_model.c:686-694).  With
libq35cuda in the process the prefetch uploads the FP8 weight / BF16
scale-grid pairs (a pair may span shards) and the BF16 lm_head, keyed by
those pointers: later q35_mm_fp8 / q35_mm_bf16 calls on the mapping are
cache hits (no upload) and give bit for bit what a first-touch upload gives."""
from __future__ import annotations

import ctypes as C
import json
import os
import struct
import time

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
PLAT = os.path.join(os.path.dirname(HERE), "qwen38-in-c_b200", "libq35plat.so")


def _write_st(path, tensors):
    """tensors: [(name, dtype, shape, bytes)] -> a safetensors file."""
    header, off, blobs = {}, 0, []
    for name, dtype, shape, data in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _plat():
    L = C.CDLL(PLAT)
    L.q35_plat_mmap_ro.restype, L.q35_plat_mmap_ro.argtypes = C.c_void_p, [C.c_char_p, C.POINTER(C.c_void_p)]
    L.q35_plat_mmap_prefetch.argtypes = [C.c_void_p]
    L.q35_plat_munmap.argtypes = [C.c_void_p]
    return L


def _offsets(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        h = json.loads(f.read(n))
    return {k: 8 + n + v["data_offsets"][0] for k, v in h.items() if k != "__metadata__"}


@pytest.mark.gpu
def test_preload_makes_first_calls_cache_hits(gpu, orc, tmp_path):
    import q35cu

    L = q35cu.load()
    L.q35cu_preload_bytes.restype = C.c_size_t
    L.q35cu_release_all()
    plat = _plat()
    Wg, Sg = orc.synth_fp8(11, 1000, 640)  # gate: weight and scales in shard A
    Wu, Su = orc.synth_fp8(12, 512, 384)   # up: weight in A, scale grid in B
    rng = np.random.default_rng(3)
    lm = (rng.standard_normal((300, 256)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    norm = np.ones(640, np.uint16)
    a, b = tmp_path / "model-00001-of-00002.safetensors", tmp_path / "model-00002-of-00002.safetensors"
    _write_st(a, [("model.layers.0.mlp.gate_proj.weight", "F8_E4M3", Wg.shape, Wg.tobytes()),
                  ("model.layers.0.mlp.gate_proj.weight_scale_inv", "BF16", Sg.shape, Sg.tobytes()),
                  ("model.layers.0.mlp.up_proj.weight", "F8_E4M3", Wu.shape, Wu.tobytes()),
                  ("model.norm.weight", "BF16", norm.shape, norm.tobytes()),
                  ("lm_head.weight", "BF16", lm.shape, lm.tobytes())])
    _write_st(b, [("model.layers.0.mlp.up_proj.weight_scale_inv", "BF16", Su.shape, Su.tobytes())])
    offa, offb = _offsets(a), _offsets(b)

    base_a, base_b = C.c_void_p(), C.c_void_p()
    ma = plat.q35_plat_mmap_ro(str(a).encode(), C.byref(base_a))
    mb = plat.q35_plat_mmap_ro(str(b).encode(), C.byref(base_b))
    assert ma and mb
    try:
        p0 = L.q35cu_preload_bytes()
        plat.q35_plat_mmap_prefetch(ma)  # gate uploaded; up waits for its scale grid
        assert L.q35cu_preload_bytes() - p0 == Wg.size + lm.size * 2
        plat.q35_plat_mmap_prefetch(mb)  # up completes across shards
        assert L.q35cu_preload_bytes() - p0 == Wg.size + lm.size * 2 + Wu.size
        resident = L.q35cu_cache_bytes()

        def ptr(base, off, t):
            return C.cast(C.c_void_p(base.value + off), t)

        x = orc.synth_act(21, (640,))
        y_map = np.empty(1000, np.float32)
        L.q35_mm_fp8(ptr(base_a, offa["model.layers.0.mlp.gate_proj.weight"], q35cu._u8p),
                     ptr(base_a, offa["model.layers.0.mlp.gate_proj.weight_scale_inv"], q35cu._u16p),
                     1000, 640, x.ctypes.data_as(q35cu._f32p), y_map.ctypes.data_as(q35cu._f32p))
        xu = orc.synth_act(22, (384,))
        yu_map = np.empty(512, np.float32)
        L.q35_mm_fp8(ptr(base_a, offa["model.layers.0.mlp.up_proj.weight"], q35cu._u8p),
                     ptr(base_b, offb["model.layers.0.mlp.up_proj.weight_scale_inv"], q35cu._u16p),
                     512, 384, xu.ctypes.data_as(q35cu._f32p), yu_map.ctypes.data_as(q35cu._f32p))
        xl = orc.synth_act(23, (256,))
        yl_map = np.empty(300, np.float32)
        L.q35_mm_bf16(ptr(base_a, offa["lm_head.weight"], q35cu._u16p), 300, 256,
                      xl.ctypes.data_as(q35cu._f32p), yl_map.ctypes.data_as(q35cu._f32p))
        assert L.q35cu_cache_bytes() == resident  # all three were resident: nothing uploaded
        # the same operands uploaded on first touch from host copies: bit for bit
        assert np.array_equal(y_map, q35cu.mm_fp8(Wg, Sg, x))
        assert np.array_equal(yu_map, q35cu.mm_fp8(Wu, Su, xu))
        assert np.array_equal(yl_map, q35cu.mm_bf16(lm, xl))

        # Q35_PRELOAD=0 keeps first-touch uploads
        os.environ["Q35_PRELOAD"] = "0"
        try:
            p1 = L.q35cu_preload_bytes()
            plat.q35_plat_mmap_prefetch(ma)
            assert L.q35cu_preload_bytes() == p1
        finally:
            del os.environ["Q35_PRELOAD"]
    finally:
        plat.q35_plat_munmap(ma)
        plat.q35_plat_munmap(mb)
        L.q35cu_release_all()


@pytest.mark.gpu
def test_preload_throughput(gpu, orc, tmp_path):
    """One ~1.1 GB shard of 17408 x 5120 FP8 weights (page cache warm):
    the prefetch's page-in plus upload, in GB/s (reported, not a bound)."""
    import q35cu

    L = q35cu.load()
    L.q35cu_preload_bytes.restype = C.c_size_t
    L.q35cu_release_all()
    plat = _plat()
    W, S = orc.synth_fp8(5, 17408, 5120)
    path = tmp_path / "big.safetensors"
    n = 12
    _write_st(path, [item for i in range(n) for item in
                     ((f"model.layers.{i}.mlp.gate_proj.weight", "F8_E4M3", W.shape, W.tobytes()),
                      (f"model.layers.{i}.mlp.gate_proj.weight_scale_inv", "BF16", S.shape, S.tobytes()))])
    base = C.c_void_p()
    m = plat.q35_plat_mmap_ro(str(path).encode(), C.byref(base))
    assert m
    try:
        p0 = L.q35cu_preload_bytes()
        t0 = time.perf_counter()
        plat.q35_plat_mmap_prefetch(m)
        dt = time.perf_counter() - t0
        assert L.q35cu_preload_bytes() - p0 == n * W.size
        print(f"preload: {n * W.size / 1e9:.2f} GB in {dt:.3f} s = {n * W.size / dt / 1e9:.1f} GB/s")
    finally:
        plat.q35_plat_munmap(m)
        L.q35cu_release_all()
