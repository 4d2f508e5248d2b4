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


def test_call_flags_match_header():
    """The per-call flag bits of the binding equal the header's."""
    text = HEADER.read_text()
    for name, bit in (("FU_FWD_SINGLE", 12), ("FU_FWD_NO_RETILE", 14),
                      ("FU_FWD_FP32_EPILOGUE", 15), ("FU_FWD_NO_PDL", 17),
                      ("FU_FWD_STATIC_WEIGHTS", 18)):
        assert re.search(rf"#define {name} \(1u << {bit}\)", text), name
        assert getattr(_C, name) == 1 << bit, name
    assert re.search(r"#define FU_FWD_PAIR \(2u << 12\)", text) and _C.FU_FWD_PAIR == 2 << 12
    assert re.search(r"#define FU_FWD_NO_PEER_WAIT 1u", text) and _C.FU_FWD_NO_PEER_WAIT == 1
    assert all(_C.FU_FWD_SPLITS(n) == (n & 0xF) << 8 for n in range(16))


def test_oproj_constants_and_errors_without_gpu():
    text = HEADER.read_text()
    assert re.search(r"#define FU_OPROJ_READY FU_SYNC_WORDS", text)
    assert _C.FU_OPROJ_READY == _C.FU_SYNC_WORDS
    for name, bit in (("FU_OPROJ_GATHER_ONLY", 20), ("FU_OPROJ_GEMM_ONLY", 21)):
        assert re.search(rf"#define {name} \(1u << {bit}\)", text), name
        assert getattr(_C, name) == 1 << bit
    # 64 words of flags and counters, then one ready counter per 128-row m-block.
    assert _C.oproj_sync_words(1) == _C.FU_SYNC_WORDS + 1
    assert _C.oproj_sync_words(4096) == _C.FU_SYNC_WORDS + 32
    assert _C.oproj_sync_words(0) == 0
    handle = ctypes.c_void_p()
    assert _C.lib.fu_oproj_create(None, ctypes.byref(handle)) == _C.FU_ERR_INVALID
    t = _C.OprojTopology()
    t.sp_size, t.sp_rank, t.q_heads, t.hidden_size, t.max_local_tokens = 2, 0, 5, 512, 8
    assert _C.lib.fu_oproj_create(ctypes.byref(t), ctypes.byref(handle)) == _C.FU_ERR_INVALID
    assert "multiple of 2" in _C.last_error()
    t.q_heads, t.hidden_size = 4, 320
    assert _C.lib.fu_oproj_create(ctypes.byref(t), ctypes.byref(handle)) == _C.FU_ERR_INVALID
    assert "hidden_size" in _C.last_error()
    t.hidden_size = 512
    assert _C.lib.fu_oproj_create(ctypes.byref(t), ctypes.byref(handle)) == _C.FU_ERR_INVALID
    assert "missing buffer" in _C.last_error()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no host C compiler")
@pytest.mark.parametrize("cname,struct", [("fu_qkv_topology", "Topology"),
                                          ("fu_oproj_topology", "OprojTopology")])
def test_topology_struct_layout(tmp_path, cname, struct):
    py = getattr(_C, struct)
    fields = [f[0] for f in py._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"',
           "int main(void) {", f'printf("size %zu\\n", sizeof({cname}));']
    for f in fields:
        src.append(f'printf("{f} %zu\\n", offsetof({cname}, {f}));')
    src += ["return 0;", "}"]
    c = tmp_path / "probe.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", str(c), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True,
                                                       capture_output=True,
                                                       text=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(py)
    for f in fields:
        assert int(out[f]) == getattr(py, f).offset, f


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no host C compiler")
def test_c_caller_links_and_calls_the_abi(tmp_path):
    """A plain C program includes the header, links the library and calls the
    entry points that need no GPU: version, argument checking and its error
    channel, sizes."""
    src = tmp_path / "caller.c"
    src.write_text(f"""
#include <stdio.h>
#include <string.h>
#include "{HEADER}"
int main(void) {{
    fu_qkv_ctx* q = NULL;
    fu_oproj_ctx* o = NULL;
    if (fu_version() < 1) return 1;
    if (fu_qkv_create(NULL, &q) != FU_ERR_INVALID || q != NULL) return 2;
    if (strstr(fu_last_error(), "null") == NULL) return 3;
    if (fu_oproj_create(NULL, &o) != FU_ERR_INVALID) return 4;
    if (fu_oproj_sync_words(4096) != FU_OPROJ_READY + 32) return 5;
    if (fu_qkv_forward(NULL, NULL, NULL, NULL, NULL, NULL, NULL, 1, 1, 1e-6, 1e-6, 0,
                       NULL, NULL) != FU_ERR_INVALID) return 6;
    printf("ok %d\\n", fu_version());
    return 0;
}}
""")
    exe = tmp_path / "caller"
    lib_dir = str(_C.LIB_PATH.parent)
    subprocess.run(["gcc", "-std=c11", str(src), "-L", lib_dir, f"-l:{_C.LIB_PATH.name}",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok ")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no host C compiler")
def test_c_example_layer_compiles(tmp_path):
    """The C example caller (one layer: forward exchange, then the output
    side) compiles against the header without warnings."""
    example = Path(__file__).resolve().parent / "c_example_layer.c"
    src = tmp_path / "example.c"
    src.write_text(example.read_text().replace('#include "flash_ulysses_b200.h"',
                                               f'#include "{HEADER}"'))
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-c", str(src),
                    "-o", str(tmp_path / "example.o")], check=True)
