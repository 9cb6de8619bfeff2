"""Python mirror of libq35cuda's C-ABI (include/q35_mm.h, include/q35cu.h).

This is the host-side view the tests and the benchmark use.  It does not
compute anything itself: every call goes through ``ctypes`` into
``libq35cuda.so`` (built in-tree by ``make`` in this directory), which
launches the sm_100a kernels.  There is no CPU fallback -- if the library is
missing, ``load()`` raises.

Two layers, mirroring the two headers:

* ``mm_fp8 / mm_fp8_batch / mm_fp8_multi4 / mm_bf16`` -- the reference's
  own entry points (qwen35-c/include/q35/q35_mm.h:24-45), called with numpy
  HOST arrays, exactly as the engine calls them.
* ``Weight`` + ``gemv / multi / gemm`` -- device-resident weights and
  device-pointer launches on a caller stream (torch tensors' data pointers),
  for the benchmark, CUDA graphs and tensor parallelism.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libq35cuda.so")
REPO = os.path.dirname(HERE)

OK, ERR_ARG, ERR_NOMEM, ERR_CUDA, ERR_UNSUPPORTED, ERR_NCCL, ERR_NODEV, ERR_TIMEOUT = range(8)
ON_ERROR_ABORT, ON_ERROR_RECORD = 0, 1
SHARD_COLUMN, SHARD_ROW = 0, 1

_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)
_vp = C.c_void_p
_u32 = C.c_uint32

# (name, restype, argtypes) for every function the headers declare
_SIGS = [
    ("q35_mm_init", None, []),
    ("q35_mm_e4m3_to_f32", C.c_float, [C.c_uint8]),
    ("q35_mm_bf16_to_f32", C.c_float, [C.c_uint16]),
    ("q35_mm_fp8", None, [_u8p, _u16p, _u32, _u32, _f32p, _f32p]),
    ("q35_mm_fp8_batch", None, [_u8p, _u16p, _u32, _u32, _u32, _f32p, _f32p]),
    ("q35_mm_fp8_multi4", None, [C.POINTER(_u8p), C.POINTER(_u16p), C.POINTER(_u32), _u32, _f32p,
                                 C.POINTER(_f32p)]),
    ("q35_mm_bf16", None, [_u16p, _u32, _u32, _f32p, _f32p]),
    ("q35_mm_impl_fp8", C.c_char_p, []),
    ("q35cu_last_error", C.c_int, []),
    ("q35cu_last_error_message", C.c_char_p, []),
    ("q35cu_clear_error", None, []),
    ("q35cu_set_error_mode", None, [C.c_int]),
    ("q35cu_get_error_mode", C.c_int, []),
    ("q35cu_device_count", C.c_int, []),
    ("q35cu_set_device", C.c_int, [C.c_int]),
    ("q35cu_sm_count", C.c_int, []),
    ("q35cu_cache_bytes", C.c_size_t, []),
    ("q35cu_set_memory_budget", None, [C.c_size_t]),
    ("q35cu_release_all", None, []),
    ("q35cu_forget", C.c_int, [_vp]),
    ("q35cu_weight_upload_fp8", C.c_int, [_u8p, _u16p, _u32, _u32, C.POINTER(_vp)]),
    ("q35cu_weight_upload_fp8_window", C.c_int, [_u8p, _u16p, _u32, _u32, _u32, _u32, _u32, _u32,
                                                 C.POINTER(_vp)]),
    ("q35cu_weight_upload_bf16", C.c_int, [_u16p, _u32, _u32, C.POINTER(_vp)]),
    ("q35cu_weight_synth_fp8", C.c_int, [C.c_uint64, C.c_float, _u32, _u32, _u32, _u32, _u32, _u32,
                                         C.POINTER(_vp)]),
    ("q35cu_weight_download_fp8", C.c_int, [_vp, _u8p, _u16p]),
    ("q35cu_weight_bind", C.c_int, [_u8p, _u16p, _vp]),
    ("q35cu_weight_free", None, [_vp]),
    ("q35cu_weight_rows", _u32, [_vp]),
    ("q35cu_weight_cols", _u32, [_vp]),
    ("q35cu_weight_device_bytes", C.c_size_t, [_vp]),
    ("q35cu_gemv_fp8", C.c_int, [_vp, _vp, _u32, _u32, _vp, _u32, _vp]),
    ("q35cu_multi_fp8", C.c_int, [C.POINTER(_vp), _vp, _u32, _u32, C.POINTER(_vp), _vp]),
    ("q35cu_gemm_fp8_workspace_bytes", C.c_size_t, [_u32, _u32]),
    ("q35cu_gemv_fp8_tc_workspace_bytes", C.c_size_t, [_u32, _u32]),
    ("q35cu_gemv_fp8_tc", C.c_int, [_vp, _vp, _u32, _vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemm_fp8", C.c_int, [_vp, _vp, _u32, _vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemm_fp8_f32", C.c_int, [_vp, _vp, _u32, _vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemm_fp8_multi", C.c_int, [_vp, _u32, _vp, C.c_int, _u32, _vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemm_fp8_f32_noalloc", C.c_int, [_vp, _vp, _u32, _vp, _vp]),
    ("q35cu_f32_to_bf16", C.c_int, [_vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemm_reserve_sms", C.c_int, [C.c_int]),
    ("q35cu_swiglu", C.c_int, [_vp, _vp, _vp, C.c_size_t, _vp]),
    ("q35cu_gemv_bf16", C.c_int, [_vp, _vp, _vp, _vp]),
    ("q35cu_shard_window", C.c_int, [_u32, _u32, C.c_int, C.c_int, C.c_int, C.POINTER(_u32),
                                     C.POINTER(_u32), C.POINTER(_u32), C.POINTER(_u32)]),
    ("q35cu_nccl_unique_id", C.c_int, [_vp, C.c_size_t]),
    ("q35cu_tp_init", C.c_int, [C.c_int, C.c_int, _vp, C.c_size_t]),
    ("q35cu_tp_world", C.c_int, []),
    ("q35cu_tp_rank", C.c_int, []),
    ("q35cu_tp_finalize", C.c_int, []),
    ("q35cu_allreduce_f32", C.c_int, [_vp, C.c_size_t, _vp]),
    ("q35cu_allgather_f32", C.c_int, [_vp, _vp, C.c_size_t, _vp]),
    ("q35cu_p2p_handle", C.c_int, [_vp, C.c_size_t]),
    ("q35cu_p2p_open", C.c_int, [C.c_int, C.c_int, _vp, C.c_size_t]),
    ("q35cu_p2p_close", C.c_int, []),
    ("q35cu_p2p_max_elems", C.c_size_t, []),
    ("q35cu_p2p_allreduce_f32", C.c_int, [_vp, _vp, C.c_size_t, _vp]),
    ("q35cu_p2p_allgather_f32", C.c_int, [_vp, _vp, C.c_size_t, _vp]),
    ("q35cu_multi_fp8_tp", C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp]),
    ("q35cu_gemv_fp8_tp", C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp]),
    ("q35cu_chain_create", C.c_int, [C.POINTER(_vp)]),
    ("q35cu_chain_add", C.c_int, [_vp, _vp, _vp, _vp, C.c_int, _vp]),
    ("q35cu_chain_run", C.c_int, [_vp, _vp]),
    ("q35cu_chain_free", None, [_vp]),
    ("q35cu_build_info", C.c_char_p, []),
    ("q35cu_launch_count", C.c_uint64, []),
    ("q35cu_device_status", C.c_int, [C.POINTER(C.c_uint32), C.c_int]),
    ("q35cu_gemm_timeout_info", C.c_int, [C.POINTER(C.c_uint32)]),
]

_lib = None


class Q35Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libq35cuda error {code}: {msg}")
        self.code = code


def build() -> None:
    """Compile libq35cuda.so in-tree (nvcc cross-compiles sm_100a without a GPU)."""
    subprocess.run(["make", "-s", "-j8", "-C", HERE], check=True)


def load(path: str = LIB_PATH):
    """Load libq35cuda.so and declare every C signature.  Raises if missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built; run `make -C {HERE}` (or __graft_entry__.build())")
    L = C.CDLL(path)
    for name, res, args in _SIGS:
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != OK:
        L = load()
        raise Q35Error(rc, L.q35cu_last_error_message().decode(errors="replace"))


def device_status(clear: bool = True) -> int:
    """The device status words (decode GEMV, tensor-core GEMM, peer-memory
    collectives) of the current device: 0, or the status of a bounded wait
    that gave up since the last clear.  Read it after a synchronisation."""
    st = C.c_uint32(0)
    check(load().q35cu_device_status(C.byref(st), 1 if clear else 0))
    return int(st.value)


def check_device_status() -> None:
    """Raise Q35Error if a device-side wait gave up since the last check
    (the GEMM's record of where it gave up goes into the message)."""
    L = load()
    where = (C.c_uint32 * 4)()
    st = device_status(clear=False)
    if st:
        check(L.q35cu_gemm_timeout_info(where))
        device_status(clear=True)
        raise Q35Error(st, "a device-side wait gave up (GEMM record: role %d, CTA %d, block %d, thread %d)"
                       % tuple(where))


def last_error() -> tuple[int, str]:
    L = load()
    return L.q35cu_last_error(), L.q35cu_last_error_message().decode(errors="replace")


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "host arrays must be C-contiguous"
    return a.ctypes.data_as(t)


# ---------------------------------------------------------------------------
# the reference's host-pointer entry points (qwen35-c/include/q35/q35_mm.h)
# ---------------------------------------------------------------------------
def mm_fp8(W: np.ndarray, sc: np.ndarray, x: np.ndarray, y: np.ndarray | None = None) -> np.ndarray:
    rows, cols = W.shape
    y = np.empty(rows, np.float32) if y is None else y
    load().q35_mm_fp8(_p(W, _u8p), _p(sc, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
    return y


def mm_fp8_batch(W: np.ndarray, sc: np.ndarray, X: np.ndarray) -> np.ndarray:
    rows, cols = W.shape
    n = X.shape[0]
    Y = np.empty((n, rows), np.float32)
    load().q35_mm_fp8_batch(_p(W, _u8p), _p(sc, _u16p), rows, cols, n, _p(X, _f32p), _p(Y, _f32p))
    return Y


def mm_fp8_multi4(Ws, scs, x: np.ndarray):
    """Ws/scs: lists of up to 4 arrays; None (or a missing entry) = rows 0."""
    Ws = list(Ws) + [None] * (4 - len(Ws))
    scs = list(scs) + [None] * (4 - len(scs))
    cols = next(w.shape[1] for w in Ws if w is not None)
    rows = (_u32 * 4)(*[0 if w is None else w.shape[0] for w in Ws])
    outs = [np.empty(max(r, 1), np.float32) for r in rows]
    wp = (_u8p * 4)(*[_u8p() if w is None else _p(w, _u8p) for w in Ws])
    sp = (_u16p * 4)(*[_u16p() if s is None else _p(s, _u16p) for s in scs])
    yp = (_f32p * 4)(*[_p(o, _f32p) for o in outs])
    load().q35_mm_fp8_multi4(wp, sp, rows, cols, _p(x, _f32p), yp)
    return [None if w is None else o[: w.shape[0]] for w, o in zip(Ws, outs)]


def mm_bf16(W16: np.ndarray, x: np.ndarray) -> np.ndarray:
    rows, cols = W16.shape
    y = np.empty(rows, np.float32)
    load().q35_mm_bf16(_p(W16, _u16p), rows, cols, _p(x, _f32p), _p(y, _f32p))
    return y


def impl() -> str:
    return load().q35_mm_impl_fp8().decode()


def lut() -> np.ndarray:
    L = load()
    L.q35_mm_init()
    return np.ctypeslib.as_array((C.c_float * 256).in_dll(L, "q35_mm_fp8_lut")).copy()


# ---------------------------------------------------------------------------
# device-resident weights and device-pointer launches
# ---------------------------------------------------------------------------
class Weight:
    """A device-resident weight (q35cu_weight*).  Freed with ``free()``."""

    def __init__(self, handle: int):
        self.h = _vp(handle)
        L = load()
        self.rows = L.q35cu_weight_rows(self.h)
        self.cols = L.q35cu_weight_cols(self.h)
        self.nbytes = L.q35cu_weight_device_bytes(self.h)

    @classmethod
    def upload_fp8(cls, W: np.ndarray, sc: np.ndarray, window=None) -> "Weight":
        rows, cols = W.shape
        out = _vp()
        L = load()
        if window is None:
            check(L.q35cu_weight_upload_fp8(_p(W, _u8p), _p(sc, _u16p), rows, cols, C.byref(out)))
        else:
            r0, nr, c0, nc = window
            check(L.q35cu_weight_upload_fp8_window(_p(W, _u8p), _p(sc, _u16p), rows, cols, r0, nr, c0, nc,
                                                   C.byref(out)))
        return cls(out.value)

    @classmethod
    def upload_bf16(cls, W16: np.ndarray) -> "Weight":
        out = _vp()
        check(load().q35cu_weight_upload_bf16(_p(W16, _u16p), W16.shape[0], W16.shape[1], C.byref(out)))
        return cls(out.value)

    @classmethod
    def synth_fp8(cls, seed: int, grows: int, gcols: int, window=None, std: float = 0.02) -> "Weight":
        r0, nr, c0, nc = window if window is not None else (0, grows, 0, gcols)
        out = _vp()
        check(load().q35cu_weight_synth_fp8(seed, std, grows, gcols, r0, nr, c0, nc, C.byref(out)))
        return cls(out.value)

    def download_fp8(self):
        W = np.empty((self.rows, self.cols), np.uint8)
        sc = np.empty(((self.rows + 127) // 128, (self.cols + 127) // 128), np.uint16)
        check(load().q35cu_weight_download_fp8(self.h, _p(W, _u8p), _p(sc, _u16p)))
        return W, sc

    def bind(self, host_W: np.ndarray, host_sc: np.ndarray) -> None:
        check(load().q35cu_weight_bind(_p(host_W, _u8p), _p(host_sc, _u16p), self.h))

    def free(self) -> None:
        if self.h:
            load().q35cu_weight_free(self.h)
            self.h = _vp()


def _ptr(t) -> int:
    return int(t.data_ptr())


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream torch reports as handle 0


def _stream(stream) -> int:
    """The CUDA stream handle to launch on: torch's current stream by default.

    A NULL handle means "the library's own stream" to the C-ABI, so torch's
    legacy default stream (handle 0) is passed as cudaStreamLegacy instead;
    launches then land on the stream the caller's events and copies use.
    """
    if stream is None:
        import torch

        stream = torch.cuda.current_stream().cuda_stream
    elif hasattr(stream, "cuda_stream"):  # a torch.cuda.Stream
        stream = stream.cuda_stream
    s = int(stream)
    return s if s != 0 else CUDA_STREAM_LEGACY


def gemv(w: Weight, X, Y, m: int | None = None, stream=None) -> None:
    """Y[m, rows] = X[m, cols] (W.s)^T on the CUDA cores (torch tensors)."""
    m = X.shape[0] if (m is None and X.dim() == 2) else (m or 1)
    ldx = X.stride(0) if X.dim() == 2 else w.cols
    ldy = Y.stride(0) if Y.dim() == 2 else w.rows
    check(load().q35cu_gemv_fp8(w.h, _ptr(X), ldx, m, _ptr(Y), ldy, _stream(stream)))


def multi(ws, X, Ys, m: int = 1, stream=None) -> None:
    """Up to four weights sharing X in one launch; ws[i] None = skipped."""
    ws = list(ws) + [None] * (4 - len(ws))
    Ys = list(Ys) + [None] * (4 - len(Ys))
    wp = (_vp * 4)(*[None if w is None else w.h.value for w in ws])
    yp = (_vp * 4)(*[None if y is None else _ptr(y) for y in Ys])
    ldx = X.stride(0) if X.dim() == 2 else next(w.cols for w in ws if w is not None)
    check(load().q35cu_multi_fp8(wp, _ptr(X), ldx, m, yp, _stream(stream)))


def gemm_workspace_bytes(m: int, cols: int) -> int:
    return int(load().q35cu_gemm_fp8_workspace_bytes(m, cols))


def gemm(w: Weight, Xb, Y, workspace=None, stream=None) -> None:
    """Tensor-core GEMM: Y[m, rows] fp32 = Xb[m, cols] (bf16 bits, any 2-byte dtype) (W.s)^T.

    ``workspace``: a device uint8 tensor of at least gemm_workspace_bytes(m, cols)
    bytes; allocated per call when omitted."""
    assert Xb.element_size() == 2 and Xb.is_contiguous() and Y.is_contiguous()
    m = Xb.shape[0]
    need = gemm_workspace_bytes(m, w.cols)
    if workspace is None:
        import torch
        workspace = torch.empty(need, dtype=torch.uint8, device=Xb.device)
    assert workspace.numel() * workspace.element_size() >= need
    check(load().q35cu_gemm_fp8(w.h, _ptr(Xb), m, _ptr(Y), _ptr(workspace),
                                workspace.numel() * workspace.element_size(), _stream(stream)))


def gemm_f32(w: Weight, X, Y, workspace=None, stream=None) -> None:
    """gemm() on fp32 activations X[m, cols] (device), rounded to bf16 as they
    are prepared: the same results as gemm(w, bf16(X), Y)."""
    assert X.dtype.itemsize == 4 and X.is_contiguous() and Y.is_contiguous()
    m = X.shape[0]
    need = gemm_workspace_bytes(m, w.cols)
    if workspace is None:
        import torch
        workspace = torch.empty(need, dtype=torch.uint8, device=X.device)
    assert workspace.numel() * workspace.element_size() >= need
    check(load().q35cu_gemm_fp8_f32(w.h, _ptr(X), m, _ptr(Y), _ptr(workspace),
                                    workspace.numel() * workspace.element_size(), _stream(stream)))


def gemm_multi(ws, X, Ys, workspace=None, stream=None) -> None:
    """Up to four GEMMs on the same activations in one launch: Ys[i][m, rows_i]
    = X[m, cols] (W_i.s)^T.  X is bf16 bits (any 2-byte dtype) or fp32 (rounded
    to bf16); the weights share cols.  Bit-identical to gemm()/gemm_f32() per weight."""
    assert 1 <= len(ws) == len(Ys) <= 4 and X.is_contiguous() and all(y.is_contiguous() for y in Ys)
    assert X.element_size() in (2, 4)
    m = X.shape[0]
    need = gemm_workspace_bytes(m, ws[0].cols)
    if workspace is None:
        import torch
        workspace = torch.empty(need, dtype=torch.uint8, device=X.device)
    assert workspace.numel() * workspace.element_size() >= need
    wp = (_vp * len(ws))(*[w.h.value for w in ws])
    yp = (_vp * len(Ys))(*[_ptr(y) for y in Ys])
    check(load().q35cu_gemm_fp8_multi(wp, len(ws), _ptr(X), int(X.element_size() == 4), m, yp, _ptr(workspace),
                                      workspace.numel() * workspace.element_size(), _stream(stream)))


def gemv_tc(w: Weight, X, Y, workspace=None, stream=None) -> None:
    """Multi-token decode on the tensor cores, exact fp32 activations (hi/lo split)."""
    assert X.dtype.itemsize == 4 and X.is_contiguous() and Y.is_contiguous()
    m = X.shape[0]
    need = int(load().q35cu_gemv_fp8_tc_workspace_bytes(m, w.cols))
    if workspace is None:
        import torch
        workspace = torch.empty(need, dtype=torch.uint8, device=X.device)
    check(load().q35cu_gemv_fp8_tc(w.h, _ptr(X), m, _ptr(Y), _ptr(workspace),
                                   workspace.numel() * workspace.element_size(), _stream(stream)))


def f32_to_bf16(x, y, stream=None) -> None:
    check(load().q35cu_f32_to_bf16(_ptr(x), _ptr(y), x.numel(), _stream(stream)))


def swiglu(g, u, o, stream=None) -> None:
    check(load().q35cu_swiglu(_ptr(g), _ptr(u), _ptr(o), g.numel(), _stream(stream)))


def gemv_bf16(w: Weight, x, y, stream=None) -> None:
    check(load().q35cu_gemv_bf16(w.h, _ptr(x), _ptr(y), _stream(stream)))


# ---------------------------------------------------------------------------
# tensor parallel
# ---------------------------------------------------------------------------
def shard_window(rows: int, cols: int, mode: int, rank: int, world: int):
    r0, nr, c0, nc = _u32(), _u32(), _u32(), _u32()
    check(load().q35cu_shard_window(rows, cols, mode, rank, world, C.byref(r0), C.byref(nr), C.byref(c0),
                                    C.byref(nc)))
    return r0.value, nr.value, c0.value, nc.value


def _torch_nccl_first() -> None:
    """libq35cuda resolves NCCL at run time and reuses a NCCL already in the
    process.  torch links its own (newer) NCCL under the same soname, so it
    must be imported before the library loads one."""
    import torch  # noqa: F401


def nccl_unique_id() -> bytes:
    _torch_nccl_first()
    buf = C.create_string_buffer(128)
    check(load().q35cu_nccl_unique_id(buf, 128))
    return buf.raw


def tp_init(rank: int, world: int, uid: bytes) -> None:
    _torch_nccl_first()
    buf = C.create_string_buffer(uid, len(uid))
    check(load().q35cu_tp_init(rank, world, buf, len(uid)))


def tp_finalize() -> None:
    check(load().q35cu_tp_finalize())


def allreduce(buf, stream=None) -> None:
    check(load().q35cu_allreduce_f32(_ptr(buf), buf.numel(), _stream(stream)))


def allgather(send, recv, stream=None) -> None:
    check(load().q35cu_allgather_f32(_ptr(send), _ptr(recv), send.numel(), _stream(stream)))


P2P_HANDLE_BYTES = 64


def p2p_handle() -> bytes:
    """Allocate this rank's NVLink exchange area; its CUDA IPC handle."""
    buf = C.create_string_buffer(P2P_HANDLE_BYTES)
    check(load().q35cu_p2p_handle(buf, P2P_HANDLE_BYTES))
    return buf.raw


def p2p_open(rank: int, world: int, handles: list) -> None:
    """Map every rank's exchange area (handles in rank order)."""
    blob = b"".join(handles)
    buf = C.create_string_buffer(blob, len(blob))
    check(load().q35cu_p2p_open(rank, world, buf, P2P_HANDLE_BYTES))


def p2p_close() -> None:
    check(load().q35cu_p2p_close())


def p2p_allreduce(buf, out=None, stream=None) -> None:
    out = buf if out is None else out
    check(load().q35cu_p2p_allreduce_f32(_ptr(buf), _ptr(out), buf.numel(), _stream(stream)))


def p2p_allgather(send, recv, stream=None) -> None:
    check(load().q35cu_p2p_allgather_f32(_ptr(send), _ptr(recv), send.numel(), _stream(stream)))


TP_ALLREDUCE, TP_ALLGATHER = 1, 2


def multi_tp(ws, X, Ys, mode: int, gathered=None, stream=None) -> None:
    """One-token decode GEMV of up to four weights with the TP exchange fused in."""
    ws = list(ws) + [None] * (4 - len(ws))
    Ys = list(Ys) + [None] * (4 - len(Ys))
    wp = (_vp * 4)(*[None if w is None else w.h.value for w in ws])
    yp = (_vp * 4)(*[None if y is None else _ptr(y) for y in Ys])
    check(load().q35cu_multi_fp8_tp(wp, _ptr(X), yp, mode, None if gathered is None else _ptr(gathered),
                                    _stream(stream)))


def gemv_tp(w, X, Y, mode: int, gathered=None, stream=None) -> None:
    multi_tp([w], X, [Y], mode, gathered, stream)


class Chain:
    """A decode chain (q35cu_chain_*): one-token GEMVs run by one cooperative launch."""

    def __init__(self):
        self.h = _vp()
        check(load().q35cu_chain_create(C.byref(self.h)))
        self._keep = []

    def add(self, ws, X, Ys, mode: int = 0, gathered=None) -> None:
        ws = list(ws) + [None] * (4 - len(ws))
        Ys = list(Ys) + [None] * (4 - len(Ys))
        wp = (_vp * 4)(*[None if w is None else w.h.value for w in ws])
        yp = (_vp * 4)(*[None if y is None else _ptr(y) for y in Ys])
        self._keep.append((X, Ys, gathered))
        check(load().q35cu_chain_add(self.h, wp, _ptr(X), yp, mode, None if gathered is None else _ptr(gathered)))

    def run(self, stream=None) -> None:
        check(load().q35cu_chain_run(self.h, _stream(stream)))

    def free(self) -> None:
        if self.h:
            load().q35cu_chain_free(self.h)
            self.h = _vp()


def declared_symbols(header: str | None = None) -> list[str]:
    """Every function/variable name declared in include/*.h (for the export
    test): the matmul library's headers by default (q35_plat.h is
    libq35plat.so's), or one named header."""
    import re

    names = []
    inc = os.path.join(REPO, "include")
    for fn in sorted(os.listdir(inc)):
        if not fn.endswith(".h") or (header is None and fn == "q35_plat.h") or (header and fn != header):
            continue
        with open(os.path.join(inc, fn)) as f:
            src = f.read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b((?:q35|q35cu)_\w+)\s*(\(|\[)", src):
            names.append(m.group(1))
    return sorted(set(names))
