"""The C-ABI library loads without a GPU, exports every function that
include/flash_ulysses_b200.h declares, and the ctypes mirror of
``fu_qkv_topology`` has the C layout (checked against a probe compiled with
the host C compiler).  No compute call is made."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from flash_ulysses_b200 import _C

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "flash_ulysses_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^FU_API\s+[\w\s\*]+?\b(fu_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "fu_qkv_forward" in names and "fu_buffer_import" in names
    assert set(names) == set(_C.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_C.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_has_sm100a_code_only_through_nvcc_build():
    from flash_ulysses_b200 import build

    assert ["-gencode", "arch=compute_100a,code=sm_100a"] == build.ARCH_FLAGS


def test_error_channel_without_gpu():
    # fu_qkv_create with a null topology fails on argument checking, before CUDA.
    handle = ctypes.c_void_p()
    rc = _C.lib.fu_qkv_create(None, ctypes.byref(handle))
    assert rc == _C.FU_ERR_INVALID
    assert "null" in _C.last_error()


def test_constants_match_header():
    text = HEADER.read_text()
    for name in ("FU_MAX_SP", "FU_HEAD_DIM", "FU_IPC_HANDLE_BYTES", "FU_SYNC_WORDS",
                 "FU_SYNC_ENTRY", "FU_SYNC_COUNTER", "FU_SYNC_EPOCH"):
        m = re.search(rf"#define {name} (\d+)", text)
        assert m and int(m.group(1)) == getattr(_C, name), name


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no host C compiler")
def test_topology_struct_layout(tmp_path):
    fields = [f[0] for f in _C.Topology._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"',
           "int main(void) {", 'printf("size %zu\\n", sizeof(fu_qkv_topology));']
    for f in fields:
        src.append(f'printf("{f} %zu\\n", offsetof(fu_qkv_topology, {f}));')
    src += ["return 0;", "}"]
    c = tmp_path / "probe.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", str(c), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True,
                                                       capture_output=True,
                                                       text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(_C.Topology)
    for f in fields:
        assert int(out[f]) == getattr(_C.Topology, f).offset, f
