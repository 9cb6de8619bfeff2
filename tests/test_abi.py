"""The C-ABI library without a GPU: it loads, exports every symbol the
headers declare, and its host-only functions behave (CPU only; no compute)."""
from __future__ import annotations

import ctypes as C
import subprocess

import numpy as np
import pytest

import q35cu


def test_library_exports_every_declared_symbol(lib):
    declared = q35cu.declared_symbols()
    assert "q35_mm_fp8" in declared and "q35_mm_fp8_lut" in declared
    out = subprocess.run(["nm", "-D", "--defined-only", q35cu.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(lib, s)


def test_platform_library_exports_every_declared_symbol():
    """include/q35_plat.h (the engine's platform layer) -> libq35plat.so."""
    import os

    declared = q35cu.declared_symbols("q35_plat.h")
    assert "q35_plat_mmap_ro" in declared and len(declared) == 27
    path = os.path.join(os.path.dirname(q35cu.LIB_PATH), "libq35plat.so")
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert not [s for s in declared if s not in exported]


def test_reference_signatures_are_unchanged():
    """q35_mm.h keeps the reference's prototypes (qwen35-c/include/q35/q35_mm.h:16-48)."""
    import os
    import re

    with open(os.path.join(q35cu.REPO, "include", "q35_mm.h")) as f:
        src = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    norm = " ".join(src.split())
    for proto in [
        "extern float q35_mm_fp8_lut[256];",
        "void q35_mm_init(void);",
        "float q35_mm_e4m3_to_f32(uint8_t v);",
        "float q35_mm_bf16_to_f32(uint16_t v);",
        "void q35_mm_fp8(const uint8_t *W, const uint16_t *scale_bf16, uint32_t rows, uint32_t cols, const float *x, float *y);",
        "void q35_mm_fp8_batch(const uint8_t *W, const uint16_t *scale_bf16, uint32_t rows, uint32_t cols, uint32_t n, const float *X, float *Y);",
        "void q35_mm_fp8_multi4(const uint8_t *W[4], const uint16_t *sc[4], uint32_t rows[4], uint32_t cols, const float *x, float *y[4]);",
        "void q35_mm_bf16(const uint16_t *W, uint32_t rows, uint32_t cols, const float *x, float *y);",
        "const char *q35_mm_impl_fp8(void);",
    ]:
        assert proto in norm, proto


def test_decoders_match_oracle(lib, orc):
    lut = q35cu.lut()
    want = orc.lut()
    assert np.array_equal(np.isnan(lut), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(lut[ok], want[ok])
    for b in range(256):
        v = lib.q35_mm_e4m3_to_f32(b)
        assert (np.isnan(v) and np.isnan(want[b])) or v == want[b]
    for h in (0, 0x3F80, 0xBF80, 0x7F80, 0x0001, 0x4049):
        assert np.float32(lib.q35_mm_bf16_to_f32(h)) == np.array([h << 16], np.uint32).view(np.float32)[0]
    assert q35cu.impl() == "sm_100a"


@pytest.mark.parametrize("rows,cols,world", [(17408, 5120, 2), (17408, 5120, 8), (5120, 17408, 8),
                                             (1024, 5120, 8), (10240, 5120, 4), (300, 260, 3)])
def test_shard_windows_tile_the_matrix(lib, rows, cols, world):
    for mode in (q35cu.SHARD_COLUMN, q35cu.SHARD_ROW):
        covered = np.zeros((rows if mode == q35cu.SHARD_COLUMN else cols,), np.int32)
        for r in range(world):
            r0, nr, c0, nc = q35cu.shard_window(rows, cols, mode, r, world)
            assert r0 % 128 == 0 and c0 % 128 == 0
            if mode == q35cu.SHARD_COLUMN:
                assert (c0, nc) == (0, cols)
                covered[r0:r0 + nr] += 1
            else:
                assert (r0, nr) == (0, rows)
                covered[c0:c0 + nc] += 1
        assert np.all(covered == 1)


def test_shard_window_rejects_bad_arguments(lib):
    with pytest.raises(q35cu.Q35Error) as e:
        q35cu.shard_window(128, 128, q35cu.SHARD_COLUMN, 0, 2)  # one block, two ranks
    assert e.value.code == q35cu.ERR_ARG
    with pytest.raises(q35cu.Q35Error):
        q35cu.shard_window(1024, 1024, q35cu.SHARD_ROW, 3, 2)


def test_error_mode_round_trip(lib):
    old = lib.q35cu_get_error_mode()
    lib.q35cu_set_error_mode(q35cu.ON_ERROR_RECORD)
    assert lib.q35cu_get_error_mode() == q35cu.ON_ERROR_RECORD
    lib.q35cu_set_error_mode(old)
    lib.q35cu_clear_error()
    assert q35cu.last_error() == (0, "")


def test_no_device_is_reported_not_crashed(lib):
    """Without a GPU the device calls fail with an error code (CPU box)."""
    if lib.q35cu_device_count() > 0:
        pytest.skip("a GPU is present")
    assert lib.q35cu_sm_count() == 0
    out = C.c_void_p()
    W = np.zeros((128, 128), np.uint8)
    sc = np.zeros((1, 1), np.uint16)
    rc = lib.q35cu_weight_upload_fp8(W.ctypes.data_as(C.POINTER(C.c_uint8)), sc.ctypes.data_as(C.POINTER(C.c_uint16)),
                                     128, 128, C.byref(out))
    assert rc == q35cu.ERR_NODEV


def test_gemm_reserve_sms_argument(lib):
    """q35cu_gemm_reserve_sms is host state only: a count of SMs the
    persistent GEMM leaves free; a negative count is refused."""
    import q35cu

    lib.q35cu_clear_error()
    assert lib.q35cu_gemm_reserve_sms(-1) == q35cu.ERR_ARG
    assert lib.q35cu_gemm_reserve_sms(16) == q35cu.OK
    assert lib.q35cu_gemm_reserve_sms(0) == q35cu.OK
