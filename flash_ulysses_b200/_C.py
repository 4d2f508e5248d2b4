"""ctypes binding of ``libflash_ulysses_b200.so`` (the C ABI in
``include/flash_ulysses_b200.h``).

Mirrors what the reference's pybind11 module ``flash_ulysses._C`` exports
(``csrc/bindings.cu:15-18``): ``launch`` and the ``TKParallelTensor`` class,
here ``ParallelTensor``.  There is no fallback: if the shared library is
missing or fails to load, importing this module raises ``ImportError``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

FU_MAX_SP = 8
FU_HEAD_DIM = 128
FU_IPC_HANDLE_BYTES = 64
FU_SYNC_WORDS = 64
FU_SYNC_ENTRY = 8
FU_SYNC_COUNTER = 32
FU_SYNC_EPOCH = 33
FU_SYNC_FAILED = 35
FU_FWD_NO_PEER_WAIT = 1


FU_FWD_SINGLE = 1 << 12
FU_FWD_PAIR = 2 << 12
FU_FWD_NO_RETILE = 1 << 14
FU_FWD_FP32_EPILOGUE = 1 << 15
FU_FWD_NO_PDL = 1 << 17
FU_FWD_STATIC_WEIGHTS = 1 << 18
FU_OPROJ_READY = FU_SYNC_WORDS
FU_OPROJ_GATHER_ONLY = 1 << 20
FU_OPROJ_GEMM_ONLY = 1 << 21


def FU_FWD_SPLITS(n):
    """Flag bits forcing the split-K factor (0 = automatic)."""
    return (n & 0xF) << 8

FU_OK, FU_ERR_INVALID, FU_ERR_CUDA, FU_ERR_UNSUPPORTED, FU_ERR_DEVICE = range(5)
STATUS_NAMES = {
    0: "ok",
    1: "pipeline wait timed out",
    2: "peer flag wait timed out",
    3: "position outside rope_cache",
}

# FLASH_ULYSSES_B200_LIB points at a library built elsewhere (e.g. a system
# install); by default the in-tree build is used.
LIB_PATH = Path(os.environ.get("FLASH_ULYSSES_B200_LIB",
                               Path(__file__).resolve().parent / "libflash_ulysses_b200.so"))

EXPORTED = (
    "fu_last_error", "fu_version",
    "fu_buffer_alloc", "fu_buffer_free", "fu_buffer_export", "fu_buffer_import",
    "fu_buffer_close", "fu_status_alloc", "fu_status_free",
    "fu_qkv_create", "fu_qkv_destroy", "fu_qkv_forward", "fu_qkv_epoch",
    "fu_qkv_last_grid", "fu_qkv_forward_noalloc",
    "fu_oproj_sync_words", "fu_oproj_create", "fu_oproj_destroy", "fu_oproj_forward",
    "fu_oproj_calls", "fu_oproj_last_grid",
)


class Topology(ctypes.Structure):
    """``fu_qkv_topology``."""

    _fields_ = [
        ("device", ctypes.c_int32),
        ("sp_size", ctypes.c_int32),
        ("sp_rank", ctypes.c_int32),
        ("q_heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("hidden_size", ctypes.c_int64),
        ("capacity_rows", ctypes.c_int64),
        ("q_recv", ctypes.c_void_p * FU_MAX_SP),
        ("k_recv", ctypes.c_void_p * FU_MAX_SP),
        ("v_recv", ctypes.c_void_p * FU_MAX_SP),
        ("sync", ctypes.c_void_p * FU_MAX_SP),
        ("status", ctypes.c_void_p),
        ("status_host", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
    ]


class OprojTopology(ctypes.Structure):
    """``fu_oproj_topology``."""

    _fields_ = [
        ("device", ctypes.c_int32),
        ("sp_size", ctypes.c_int32),
        ("sp_rank", ctypes.c_int32),
        ("q_heads", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("reserved1", ctypes.c_int32),
        ("hidden_size", ctypes.c_int64),
        ("max_local_tokens", ctypes.c_int64),
        ("gather", ctypes.c_void_p * FU_MAX_SP),
        ("sync", ctypes.c_void_p * FU_MAX_SP),
        ("status", ctypes.c_void_p),
        ("status_host", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
    ]


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m flash_ulysses_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, i32, i64, u32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32
    sig = {
        "fu_last_error": (ctypes.c_char_p, []),
        "fu_version": (ctypes.c_int, []),
        "fu_buffer_alloc": (ctypes.c_int, [ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "fu_buffer_free": (ctypes.c_int, [ctypes.c_int, vp]),
        "fu_buffer_export": (ctypes.c_int, [ctypes.c_int, vp, ctypes.c_char_p]),
        "fu_buffer_import": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(vp)]),
        "fu_buffer_close": (ctypes.c_int, [ctypes.c_int, vp]),
        "fu_status_alloc": (ctypes.c_int, [ctypes.POINTER(vp), ctypes.POINTER(vp)]),
        "fu_status_free": (ctypes.c_int, [vp]),
        "fu_qkv_create": (ctypes.c_int, [ctypes.POINTER(Topology), ctypes.POINTER(vp)]),
        "fu_qkv_destroy": (ctypes.c_int, [vp]),
        "fu_qkv_forward": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, vp, i64, i64,
                                          ctypes.c_double, ctypes.c_double, u32, vp, vp]),
        "fu_qkv_epoch": (u32, [vp]),
        "fu_qkv_last_grid": (ctypes.c_int, [vp]),
        "fu_qkv_forward_noalloc": (ctypes.c_int, [ctypes.c_int, vp, vp, vp, vp, vp, vp, i64, i64,
                                                  i32, i32, i64, ctypes.c_double,
                                                  ctypes.c_double, vp, vp, vp, vp, vp]),
        "fu_oproj_sync_words": (i64, [i64]),
        "fu_oproj_create": (ctypes.c_int, [ctypes.POINTER(OprojTopology), ctypes.POINTER(vp)]),
        "fu_oproj_destroy": (ctypes.c_int, [vp]),
        "fu_oproj_forward": (ctypes.c_int, [vp, vp, vp, i64, vp, u32, vp]),
        "fu_oproj_calls": (u32, [vp]),
        "fu_oproj_last_grid": (ctypes.c_int, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# The CPython fast-call binding of fu_qkv_forward, when it was built against
# the library in use (it links the in-tree build).
try:
    if "FLASH_ULYSSES_B200_LIB" in os.environ:
        raise ImportError("library path overridden")
    from . import _fu_fast as _fast
except ImportError:
    _fast = None

_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream_handle(device_index):
    """The cudaStream_t of the current torch stream on `device_index`."""
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def last_error():
    return lib.fu_last_error().decode(errors="replace")


def check(rc, what):
    if rc != FU_OK:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")


def decode_status(word):
    code, where = word & 0xFF, (word >> 8) & 0xFF
    return f"{STATUS_NAMES.get(code, f'status {code}')} (site {where})"


class _DeviceMemory:
    """Exposes a raw device allocation through ``__cuda_array_interface__`` so
    torch can view it without copying."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {
            "shape": (nbytes // 2,),
            "typestr": "<i2",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }


def tensor_from_device_ptr(ptr, shape, dtype, device):
    """A torch tensor aliasing ``ptr`` (which this process must own)."""
    nbytes = 1
    for s in shape:
        nbytes *= s
    nbytes *= torch.empty((), dtype=dtype).element_size()
    with torch.cuda.device(device):
        flat = torch.as_tensor(_DeviceMemory(ptr, nbytes), device=device)
    return flat.view(dtype).view(*shape)


class ParallelTensor:
    """A receive buffer allocated by every rank and mapped by its peers.

    Mirrors ThunderKittens' ``TKParallelTensor(shape, dtype, rank, world,
    multicast)`` as used by the reference (context.py:63-90): ``data_`` is the
    full local tensor, ``data()`` returns it, ``local_rank_`` and
    ``local_world_size_`` describe the world.  Construction is collective over
    ``group``: the 64-byte CUDA IPC handles are exchanged with
    ``all_gather_object`` and every rank maps the handles of ``peers``
    (global ranks; default: the whole world).  ``peer_ptr(r)`` is rank r's
    buffer as seen from this process.  NVLink multicast is not used
    (``multicast`` must be False).
    """

    def __init__(self, shape, dtype, rank, world_size, multicast=False, *, group=None,
                 peers=None, device=None):
        if multicast:
            raise ValueError("multicast parallel tensors are not used by this build")
        self.local_rank_ = rank
        self.local_world_size_ = world_size
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device(device).index)
        self.shape = tuple(shape)
        self.dtype = dtype
        numel = 1
        for s in self.shape:
            numel *= s
        nbytes = max(numel * torch.empty((), dtype=dtype).element_size(), 256)
        ptr = ctypes.c_void_p()
        check(lib.fu_buffer_alloc(self.device.index, nbytes, ctypes.byref(ptr)), "fu_buffer_alloc")
        self._ptr = ptr.value
        self._imported = {}
        self._closed = False
        self.data_ = tensor_from_device_ptr(self._ptr, self.shape, dtype, self.device)
        peers = list(range(world_size)) if peers is None else list(peers)
        if world_size > 1:
            handle = ctypes.create_string_buffer(FU_IPC_HANDLE_BYTES)
            check(lib.fu_buffer_export(self.device.index, self._ptr, handle), "fu_buffer_export")
            handles = [None] * world_size
            torch.distributed.all_gather_object(handles, handle.raw, group=group)
            for r in peers:
                if r == rank:
                    continue
                peer = ctypes.c_void_p()
                check(lib.fu_buffer_import(self.device.index, handles[r], ctypes.byref(peer)),
                      "fu_buffer_import")
                self._imported[r] = peer.value

    def data(self):
        return self.data_

    def peer_ptr(self, r):
        return self._ptr if r == self.local_rank_ else self._imported[r]

    def close(self):
        if self._closed:
            return
        self._closed = True
        self.data_ = None
        for p in self._imported.values():
            lib.fu_buffer_close(self.device.index, p)
        self._imported = {}
        lib.fu_buffer_free(self.device.index, self._ptr)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StatusWord:
    """Host-mapped int32 the kernel writes on a device-side error."""

    def __init__(self):
        h, d = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib.fu_status_alloc(ctypes.byref(h), ctypes.byref(d)), "fu_status_alloc")
        self.host_ptr, self.device_ptr = h.value, d.value
        self._view = ctypes.cast(self.host_ptr, ctypes.POINTER(ctypes.c_int32))

    @property
    def value(self):
        return int(self._view[0])

    def clear(self):
        self._view[0] = 0

    def free(self):
        if self.host_ptr:
            lib.fu_status_free(self.host_ptr)
            self.host_ptr = None


class QkvOp:
    """Owner of one ``fu_qkv_ctx`` (the per-rank operator state)."""

    def __init__(self, topology: Topology):
        handle = ctypes.c_void_p()
        check(lib.fu_qkv_create(ctypes.byref(topology), ctypes.byref(handle)), "fu_qkv_create")
        self.handle = handle.value
        self.topology = topology

    def forward(self, x, w, positions, q_gamma, k_gamma, rope, local_tokens, rope_rows,
                q_eps, k_eps, flags=0, stream=None, gemm_out=None):
        """Launch one fused call; all tensor arguments are raw device pointers."""
        if _fast is not None:
            _fast.forward(self.handle, x, w, positions, q_gamma, k_gamma, rope, local_tokens,
                          rope_rows, q_eps, k_eps, flags, stream, gemm_out)
            return
        rc = lib.fu_qkv_forward(self.handle, x, w, positions, q_gamma, k_gamma, rope,
                                local_tokens, rope_rows, q_eps, k_eps, flags, stream, gemm_out)
        if rc != FU_OK:
            raise RuntimeError(f"fu_qkv_forward failed (code {rc}): {last_error()}")

    @property
    def epoch(self):
        return lib.fu_qkv_epoch(self.handle)

    @property
    def last_grid(self):
        return lib.fu_qkv_last_grid(self.handle)

    def destroy(self):
        if self.handle:
            lib.fu_qkv_destroy(self.handle)
            self.handle = None


class OprojOp:
    """Owner of one ``fu_oproj_ctx`` (inverse exchange + output projection)."""

    def __init__(self, topology: OprojTopology):
        handle = ctypes.c_void_p()
        check(lib.fu_oproj_create(ctypes.byref(topology), ctypes.byref(handle)),
              "fu_oproj_create")
        self.handle = handle.value
        self.topology = topology

    def forward(self, attn, w_o, local_tokens, out, flags=0, stream=None):
        """Launch one call; tensor arguments are raw device pointers."""
        rc = lib.fu_oproj_forward(self.handle, attn, w_o, local_tokens, out, flags, stream)
        if rc != FU_OK:
            raise RuntimeError(f"fu_oproj_forward failed (code {rc}): {last_error()}")

    @property
    def calls(self):
        return lib.fu_oproj_calls(self.handle)

    @property
    def last_grid(self):
        return lib.fu_oproj_last_grid(self.handle)

    def destroy(self):
        if self.handle:
            lib.fu_oproj_destroy(self.handle)
            self.handle = None


def oproj_sync_words(max_local_tokens):
    return int(lib.fu_oproj_sync_words(max_local_tokens))


def launch(x, qkv_weight, positions, q_gamma, k_gamma, rope, op: QkvOp, *, q_epsilon,
           k_epsilon, flags=0, gemm_out=None):
    """Tensor-level launch on the current stream (the role of the reference's
    ``_C.launch``, kernel_hopper.cu:305-353).  Inputs are trusted to be
    contiguous device tensors of the documented dtypes, as in the reference."""
    stream = current_stream_handle(x.get_device())
    op.forward(x.data_ptr(), qkv_weight.data_ptr(), positions.data_ptr(), q_gamma.data_ptr(),
               k_gamma.data_ptr(), rope.data_ptr(), x.shape[0], rope.shape[0], float(q_epsilon),
               float(k_epsilon), flags, stream,
               None if gemm_out is None else gemm_out.data_ptr())


__all__ = [
    "lib", "Topology", "OprojTopology", "ParallelTensor", "StatusWord", "QkvOp", "OprojOp",
    "oproj_sync_words", "launch", "check",
    "decode_status", "tensor_from_device_ptr", "EXPORTED", "LIB_PATH",
]

if os.environ.get("FLASH_ULYSSES_B200_DEBUG"):
    print(f"[flash_ulysses_b200] loaded {LIB_PATH} (ABI v{lib.fu_version()})")
