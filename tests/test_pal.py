"""The POSIX platform layer (libq35plat.so, include/q35_plat.h): every entry
point of the reference's interface (qwen35-c/src/q35_plat.h) against its
contract, on the CPU.  The reference ships only a Windows implementation
(qwen35-c/src/q35_plat_win.c) whose directory walk and file mapping are stubs
on other systems; these are the functions the engine's loader needs
(qwen35-c/src/q35_st.c, q35_model.c)."""
from __future__ import annotations

import ctypes as C
import os
import socket
import threading

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(os.path.dirname(HERE), "qwen38-in-c_b200", "libq35plat.so")


@pytest.fixture(scope="module")
def pal():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (make -C qwen38-in-c_b200)")
    L = C.CDLL(LIB)
    vp, sz = C.c_void_p, C.c_size_t
    sigs = {
        "q35_plat_read_file": (vp, [C.c_char_p, C.POINTER(sz)]),
        "q35_plat_aligned_alloc": (vp, [sz, sz]),
        "q35_plat_aligned_free": (None, [vp]),
        "q35_plat_large_alloc": (vp, [sz]),
        "q35_plat_large_free": (None, [vp]),
        "q35_plat_free": (None, [vp]),
        "q35_plat_now": (C.c_double, []),
        "q35_plat_dir_open": (vp, [C.c_char_p]),
        "q35_plat_dir_next": (C.c_char_p, [vp]),
        "q35_plat_dir_close": (None, [vp]),
        "q35_plat_fseek64": (C.c_int, [vp, C.c_int64, C.c_int]),
        "q35_plat_ftell64": (C.c_int64, [vp]),
        "q35_plat_mmap_ro": (vp, [C.c_char_p, C.POINTER(vp)]),
        "q35_plat_munmap": (None, [vp]),
        "q35_plat_mmap_prefetch": (None, [vp]),
        "q35_plat_avail_phys": (C.c_uint64, []),
        "q35_plat_peak_rss": (sz, []),
        "q35_plat_num_phys_cores": (C.c_int, []),
        "q35_plat_strdup": (vp, [C.c_char_p]),
        "q35_plat_path_join": (C.c_int, [C.c_char_p, sz, C.c_char_p, C.c_char_p]),
        "q35_plat_prefetch": (None, [vp, sz]),
        "q35_plat_sock_init": (C.c_int, []),
        "q35_plat_sock_listen": (C.c_int, [C.c_int]),
        "q35_plat_sock_accept": (C.c_int, [C.c_int]),
        "q35_plat_sock_recv": (C.c_int, [C.c_int, vp, sz]),
        "q35_plat_sock_send": (C.c_int, [C.c_int, vp, sz]),
        "q35_plat_sock_close": (None, [C.c_int]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(L, name)  # every entry point of the interface is exported
        f.restype, f.argtypes = res, args
    return L


def test_read_file(pal, tmp_path):
    p = tmp_path / "blob.bin"
    data = bytes(range(256)) * 37
    p.write_bytes(data)
    n = C.c_size_t(0)
    buf = pal.q35_plat_read_file(str(p).encode(), C.byref(n))
    assert buf and n.value == len(data)
    assert C.string_at(buf, n.value) == data and C.string_at(buf + n.value, 1) == b"\0"  # NUL-terminated
    pal.q35_plat_free(buf)
    e = tmp_path / "empty"
    e.write_bytes(b"")
    buf = pal.q35_plat_read_file(str(e).encode(), C.byref(n))
    assert buf and n.value == 0
    pal.q35_plat_free(buf)
    n.value = 12345
    assert not pal.q35_plat_read_file(str(tmp_path / "missing").encode(), C.byref(n))
    assert n.value == 12345  # untouched on failure


def test_allocators(pal):
    for align in (16, 64, 4096):
        p = pal.q35_plat_aligned_alloc(align, 1000)
        assert p and p % align == 0
        C.memset(p, 7, 1000)
        pal.q35_plat_aligned_free(p)
    assert not pal.q35_plat_large_alloc(4096)  # below one huge page: the caller's own allocator
    big = 8 << 20
    p = pal.q35_plat_large_alloc(big)
    if p:  # a huge-page (or transparent-huge-page) mapping, writable end to end
        C.memset(p, 1, big)
        assert C.string_at(p + big - 4, 4) == b"\x01" * 4
        pal.q35_plat_large_free(p)
    pal.q35_plat_large_free(None)


def test_now_monotonic(pal):
    a = pal.q35_plat_now()
    b = pal.q35_plat_now()
    assert b >= a > 0


def test_dir_regular_files_only(pal, tmp_path):
    for n in ("b.safetensors", "a.json"):
        (tmp_path / n).write_bytes(b"x")
    (tmp_path / "sub").mkdir()
    os.symlink(tmp_path / "a.json", tmp_path / "link.json")
    d = pal.q35_plat_dir_open(str(tmp_path).encode())
    assert d
    names = []
    while True:
        s = pal.q35_plat_dir_next(d)
        if s is None:
            break
        names.append(s.decode())
    pal.q35_plat_dir_close(d)
    assert sorted(names) == ["a.json", "b.safetensors", "link.json"]  # no ".", "..", "sub"
    assert not pal.q35_plat_dir_open(str(tmp_path / "nope").encode())
    assert pal.q35_plat_dir_next(None) is None


def test_seek_tell_64bit(pal, tmp_path):
    libc = C.CDLL(None)
    libc.fopen.restype, libc.fopen.argtypes = C.c_void_p, [C.c_char_p, C.c_char_p]
    libc.fclose.argtypes = [C.c_void_p]
    p = tmp_path / "sparse"
    with open(p, "wb") as f:
        f.truncate(5 << 30)  # sparse: no blocks written
    fp = libc.fopen(str(p).encode(), b"rb")
    assert fp
    off = (4 << 30) + 12345  # beyond 32-bit offsets
    assert pal.q35_plat_fseek64(fp, off, 0) == 0
    assert pal.q35_plat_ftell64(fp) == off
    assert pal.q35_plat_fseek64(fp, 0, 2) == 0 and pal.q35_plat_ftell64(fp) == 5 << 30
    libc.fclose(fp)


def test_mmap_ro(pal, tmp_path):
    p = tmp_path / "w.bin"
    data = os.urandom(3 * 4096 + 17)
    p.write_bytes(data)
    base = C.c_void_p()
    m = pal.q35_plat_mmap_ro(str(p).encode(), C.byref(base))
    assert m and base.value
    pal.q35_plat_mmap_prefetch(m)
    assert C.string_at(base.value, len(data)) == data
    pal.q35_plat_prefetch(base.value + 5, 100)
    pal.q35_plat_prefetch(None, 0)
    pal.q35_plat_munmap(m)
    pal.q35_plat_munmap(None)
    (tmp_path / "empty").write_bytes(b"")
    assert not pal.q35_plat_mmap_ro(str(tmp_path / "empty").encode(), C.byref(base))
    assert not pal.q35_plat_mmap_ro(str(tmp_path / "missing").encode(), C.byref(base))


def test_system_queries(pal):
    assert pal.q35_plat_avail_phys() > 0
    assert pal.q35_plat_peak_rss() > 1 << 20  # this Python process
    n = pal.q35_plat_num_phys_cores()
    assert 1 <= n <= (os.cpu_count() or n)


def test_strings(pal):
    s = pal.q35_plat_strdup(b"q35")
    assert C.string_at(s) == b"q35"
    pal.q35_plat_free(s)
    buf = C.create_string_buffer(16)
    assert pal.q35_plat_path_join(buf, 16, b"dir", b"file") == 0 and buf.value == b"dir/file"
    assert pal.q35_plat_path_join(buf, 8, b"dir", b"file") == -1  # does not fit


def test_loopback_socket(pal):
    assert pal.q35_plat_sock_init() == 0
    with socket.socket() as s:  # a free port
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    lfd = pal.q35_plat_sock_listen(port)
    assert lfd >= 0
    got = {}

    def client():
        with socket.create_connection(("127.0.0.1", port), timeout=10) as c:
            c.sendall(b"GET /health")
            got["reply"] = c.recv(64)

    th = threading.Thread(target=client)
    th.start()
    fd = pal.q35_plat_sock_accept(lfd)
    assert fd >= 0
    buf = C.create_string_buffer(64)
    n = pal.q35_plat_sock_recv(fd, buf, 64)
    assert buf.raw[:n] == b"GET /health"
    msg = b"ok"
    assert pal.q35_plat_sock_send(fd, msg, len(msg)) == len(msg)
    th.join(10)
    pal.q35_plat_sock_close(fd)
    pal.q35_plat_sock_close(lfd)
    assert got.get("reply") == b"ok"
    again = pal.q35_plat_sock_listen(port)  # the port is free again at once (SO_REUSEADDR)
    assert again >= 0
    pal.q35_plat_sock_close(again)
