"""CPU oracle for the FP8 block-scaled matmul path -- TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm import this module, and only as the checker.  The product
library (``libq35cuda.so``) never touches it.

Two CPU implementations are exposed, both over numpy arrays:

* ``Oracle``     -- ``liboracle.so``, the scalar C restatement in
  ``q35_oracle.c`` (reference: qwen35-c/src/q35_mm.c:22-246), plus an fp64
  product, FNV-1a and the seeded synthetic generator.
* ``Reference``  -- ``_ref/libq35ref.so``, the unmodified reference
  ``q35_mm.c`` compiled with its symbols renamed ``ref_q35_*``.  Present when
  the reference tree was available at build time (the .so then travels with
  the repository snapshot).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libq35ref.so")
LIB_REF_SCALAR = os.path.join(HERE, "_ref", "libq35ref_scalar.so")
# the reference engine's source tree (its qwen35-c directory), if given
REFERENCE_TREE = os.environ.get("Q35_REF", "")

_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "arrays handed to the oracle must be C-contiguous"
    return a.ctypes.data_as(t)


def build(ref: bool | None = None) -> None:
    """Compile liboracle.so (and _ref/*.so when the reference tree exists)."""
    targets = ["oracle"]
    if ref or (ref is None and REFERENCE_TREE and os.path.isdir(REFERENCE_TREE)):
        targets += ["ref", f"REF={REFERENCE_TREE}"]
    subprocess.run(["make", "-s", "-C", HERE, *targets], check=True)


class Oracle:
    """ctypes view of liboracle.so (the C restatement)."""

    def __init__(self, path: str = LIB_ORACLE):
        if not os.path.exists(path):
            build(ref=False)
        L = C.CDLL(path)
        L.orc_e4m3_to_f32.restype = C.c_float
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_e4m3_rne.restype = C.c_uint8
        L.orc_f32_to_e4m3_rne.argtypes = [C.c_float]
        L.orc_f32_to_bf16_rne.restype = C.c_uint16
        L.orc_f32_to_bf16_rne.argtypes = [C.c_float]
        L.orc_lut.restype = _f32p
        L.orc_mm_fp8.argtypes = [_u8p, _u16p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.orc_mm_fp8_batch.argtypes = [_u8p, _u16p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.orc_mm_bf16.argtypes = [_u16p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.orc_mm_fp8_f64.argtypes = [_u8p, _u16p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _f64p, _f64p]
        L.orc_fnv1a.restype = C.c_uint64
        L.orc_fnv1a.argtypes = [C.c_void_p, C.c_size_t]
        L.orc_synth_normal.restype = C.c_float
        L.orc_synth_normal.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_synth_fp8.restype = C.c_int
        L.orc_synth_fp8.argtypes = [C.c_uint64, C.c_float, C.c_uint32, C.c_uint32, C.c_uint32,
                                    C.c_uint32, C.c_uint32, C.c_uint32, _u8p, _u16p]
        L.orc_synth_act.argtypes = [C.c_uint64, C.c_size_t, C.c_int, _f32p]
        L.orc_threads.restype = C.c_int
        self.L = L

    # -- decoders -------------------------------------------------------
    def lut(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.L.orc_lut(), shape=(256,)).copy()

    def e4m3_rne(self, v: float) -> int:
        return int(self.L.orc_f32_to_e4m3_rne(float(v)))

    # -- products -------------------------------------------------------
    def mm_fp8(self, W, sc, x) -> np.ndarray:
        rows, cols = W.shape
        y = np.empty(rows, np.float32)
        self.L.orc_mm_fp8(_p(W, _u8p), _p(sc, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
        return y

    def mm_fp8_batch(self, W, sc, X) -> np.ndarray:
        rows, cols = W.shape
        n = X.shape[0]
        Y = np.empty((n, rows), np.float32)
        self.L.orc_mm_fp8_batch(_p(W, _u8p), _p(sc, _u16p), rows, cols, n, _p(X, _f32p), _p(Y, _f32p))
        return Y

    def mm_bf16(self, W16, x) -> np.ndarray:
        rows, cols = W16.shape
        y = np.empty(rows, np.float32)
        self.L.orc_mm_bf16(_p(W16, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
        return y

    def mm_fp8_f64(self, W, sc, X):
        """(Y64, ABS): fp64 product and sum_k |w*s*x| per output, [n, rows]."""
        rows, cols = W.shape
        X = np.ascontiguousarray(X.reshape(-1, cols), np.float32)
        n = X.shape[0]
        Y = np.empty((n, rows), np.float64)
        A = np.empty((n, rows), np.float64)
        self.L.orc_mm_fp8_f64(_p(W, _u8p), _p(sc, _u16p), rows, cols, n, _p(X, _f32p),
                              _p(Y, _f64p), _p(A, _f64p))
        return Y, A

    def fnv1a(self, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        return int(self.L.orc_fnv1a(a.ctypes.data, a.nbytes))

    # -- synthetic data -------------------------------------------------
    def synth_fp8(self, seed: int, grows: int, gcols: int, row0: int = 0, col0: int = 0,
                  nrows: int | None = None, ncols: int | None = None, std: float = 0.02):
        nrows = grows - row0 if nrows is None else nrows
        ncols = gcols - col0 if ncols is None else ncols
        W = np.empty((nrows, ncols), np.uint8)
        sc = np.empty(((nrows + 127) // 128, (ncols + 127) // 128), np.uint16)
        rc = self.L.orc_synth_fp8(seed, std, grows, gcols, row0, col0, nrows, ncols,
                                  _p(W, _u8p), _p(sc, _u16p))
        if rc:
            raise ValueError(f"orc_synth_fp8 rejected the window (rc={rc})")
        return W, sc

    def synth_act(self, seed: int, shape, round_bf16: bool = False) -> np.ndarray:
        out = np.empty(shape, np.float32)
        self.L.orc_synth_act(seed, out.size, int(round_bf16), _p(out, _f32p))
        return out

    def threads(self) -> int:
        return int(self.L.orc_threads())


class Reference:
    """ctypes view of the unmodified reference q35_mm.c (symbols ref_q35_*)."""

    def __init__(self, path: str = LIB_REF):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        L.ref_q35_mm_init.argtypes = []
        L.ref_q35_mm_fp8.argtypes = [_u8p, _u16p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.ref_q35_mm_fp8_batch.argtypes = [_u8p, _u16p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.ref_q35_mm_fp8_multi4.argtypes = [C.POINTER(_u8p), C.POINTER(_u16p), C.POINTER(C.c_uint32),
                                            C.c_uint32, _f32p, C.POINTER(_f32p)]
        L.ref_q35_mm_bf16.argtypes = [_u16p, C.c_uint32, C.c_uint32, _f32p, _f32p]
        L.ref_q35_mm_impl_fp8.restype = C.c_char_p
        L.ref_q35_mm_init()
        self.L = L
        self.path = path

    @staticmethod
    def available(path: str = LIB_REF) -> bool:
        return os.path.exists(path)

    def impl(self) -> str:
        return self.L.ref_q35_mm_impl_fp8().decode()

    def mm_fp8(self, W, sc, x) -> np.ndarray:
        rows, cols = W.shape
        y = np.empty(rows, np.float32)
        self.L.ref_q35_mm_fp8(_p(W, _u8p), _p(sc, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
        return y

    def mm_fp8_batch(self, W, sc, X) -> np.ndarray:
        rows, cols = W.shape
        n = X.shape[0]
        Y = np.empty((n, rows), np.float32)
        self.L.ref_q35_mm_fp8_batch(_p(W, _u8p), _p(sc, _u16p), rows, cols, n, _p(X, _f32p), _p(Y, _f32p))
        return Y

    def mm_fp8_multi4(self, Ws, scs, x):
        """Ws/scs: up to 4 arrays (None = skipped segment)."""
        Ws = list(Ws) + [None] * (4 - len(Ws))
        scs = list(scs) + [None] * (4 - len(scs))
        cols = next(w.shape[1] for w in Ws if w is not None)
        rows = (C.c_uint32 * 4)(*[0 if w is None else w.shape[0] for w in Ws])
        outs = [np.empty(max(r, 1), np.float32) for r in rows]
        wp = (_u8p * 4)(*[_u8p() if w is None else _p(w, _u8p) for w in Ws])
        sp = (_u16p * 4)(*[_u16p() if s is None else _p(s, _u16p) for s in scs])
        yp = (_f32p * 4)(*[_p(o, _f32p) for o in outs])
        self.L.ref_q35_mm_fp8_multi4(wp, sp, rows, cols, _p(x, _f32p), yp)
        return [None if w is None else o[: w.shape[0]] for w, o in zip(Ws, outs)]

    def mm_bf16(self, W16, x) -> np.ndarray:
        rows, cols = W16.shape
        y = np.empty(rows, np.float32)
        self.L.ref_q35_mm_bf16(_p(W16, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
        return y


def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 value, returned as fp32 (numpy, finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 storage bits (uint16)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def dequant(W: np.ndarray, sc: np.ndarray, lut: np.ndarray) -> np.ndarray:
    """fp32 W * s (exact), for numpy-side checks."""
    rows, cols = W.shape
    s = (sc.astype(np.uint32) << 16).view(np.float32)
    s_full = np.repeat(np.repeat(s, 128, axis=0)[:rows], 128, axis=1)[:, :cols]
    return lut[W] * s_full
