"""Host logic of the collective entry points, on CPU.

NCCL is resolved at run time and every symbol is checked before the first
call, as the reference checks its run-time libraries (compute-cuda/src/
libraries.rs:100-174: a missing symbol is reported by name before any call).
These tests point FB_NCCL_LIBRARY at stand-in libraries compiled here, so no
GPU and no real NCCL is involved; each case runs in a fresh interpreter
because a successful resolution is cached for the process."""

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "forma_b200" / "libforma_b200.so"

ALL = ["ncclGetUniqueId", "ncclCommInitRank", "ncclCommInitAll", "ncclCommDestroy", "ncclCommCuDevice",
       "ncclAllReduce", "ncclGetErrorString"]


def _stand_in(tmp_path: Path, symbols) -> Path:
    """A shared library exporting `symbols`: ncclGetUniqueId writes a known
    pattern, ncclCommInitRank returns a handle that encodes (nranks, rank)."""
    body = ["#include <string.h>", "#include <stdint.h>"]
    for s in symbols:
        if s == "ncclGetUniqueId":
            body.append("int ncclGetUniqueId(char* id) { for (int i = 0; i < 128; ++i) id[i] = (char)(i * 7); return 0; }")
        elif s == "ncclCommInitRank":
            # the unique id travels by value, as ncclCommInitRank declares it
            body.append("typedef struct { char internal[128]; } uid;")
            body.append("int ncclCommInitRank(void** c, int n, uid id, int r) {"
                        " *c = (void*)(uintptr_t)(0x1000 + n * 16 + r + (unsigned char)id.internal[5]); return 0; }")
        elif s == "ncclGetErrorString":
            body.append('const char* ncclGetErrorString(int r) { return "stand-in error"; }')
        elif s == "ncclCommDestroy":
            body.append("int ncclCommDestroy(void* c) { return c == (void*)0x1 ? 3 : 0; }")
        else:
            body.append(f"int {s}() {{ return 0; }}")
    src = tmp_path / "nccl_stand_in.c"
    src.write_text("\n".join(body) + "\n")
    so = tmp_path / "libnccl_stand_in.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-o", str(so), str(src)], check=True)
    return so


def _run(code: str, nccl_library: str) -> str:
    env = dict(os.environ, FB_NCCL_LIBRARY=nccl_library)
    prog = textwrap.dedent(f"""
        import ctypes as C
        lib = C.CDLL({str(LIB)!r})
        lib.fb_last_error.restype = C.c_char_p
    """) + textwrap.dedent(code)
    r = subprocess.run([sys.executable, "-c", prog], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout.strip()


def test_missing_library_is_a_driver_error(tmp_path):
    out = _run("""
        buf = (C.c_char * 128)()
        print(lib.fb_nccl_unique_id(buf), lib.fb_last_error().decode())
    """, str(tmp_path / "no_such_libnccl.so"))
    status, detail = out.split(" ", 1)
    assert status == "34" and "NCCL is unavailable" in detail


@pytest.mark.parametrize("missing", ["ncclCommInitAll", "ncclAllReduce", "ncclGetErrorString"])
def test_missing_symbol_is_named_before_any_call(tmp_path, missing):
    so = _stand_in(tmp_path, [s for s in ALL if s != missing])
    out = _run("""
        buf = (C.c_char * 128)(*([b"x"] * 128))
        print(lib.fb_nccl_unique_id(buf), bytes(buf)[:4], lib.fb_last_error().decode())
    """, str(so))
    status, rest = out.split(" ", 1)
    assert status == "37", out
    assert rest.startswith("b'xxxx'")  # nothing was called: the buffer is untouched
    assert rest.endswith("missing symbol " + missing)


def test_complete_library_is_called(tmp_path):
    so = _stand_in(tmp_path, ALL)
    out = _run("""
        buf = (C.c_char * 128)()
        assert lib.fb_nccl_unique_id(buf) == 0
        assert bytes(buf) == bytes((i * 7) % 256 for i in range(128))
        comm = C.c_void_p()
        assert lib.fb_nccl_comm_init_rank(C.byref(comm), 4, buf, 3) == 0
        print(hex(comm.value))
        assert lib.fb_nccl_comm_init_rank(C.byref(comm), 4, buf, 4) == 32   # rank outside 0..3
        assert lib.fb_nccl_comm_destroy(C.c_void_p(1)) == 34                # the library's error, named
        print(lib.fb_last_error().decode())
        assert lib.fb_nccl_comm_destroy(None) == 0
    """, str(so))
    handle, err = out.splitlines()
    assert int(handle, 16) == 0x1000 + 4 * 16 + 3 + 35
    assert err == "ncclCommDestroy: stand-in error"
