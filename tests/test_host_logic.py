"""Host-side logic without a GPU: the constructor's validation (reference
context.py:40-60 plus this build's relaxations) and the collective exchange of
receive-buffer handles over a gloo control group, with the native buffer
calls replaced by a recording fake."""

import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_ulysses_b200 import FlashUlyssesContext


@pytest.mark.parametrize("kwargs,match", [
    (dict(world_size=4, sp_size=3), "SP must divide"),
    (dict(world_size=16, sp_size=16), "SP must divide"),
    (dict(world_size=2, sp_size=4), "SP must divide"),
    (dict(hidden_size=100), "divisible by 64"),
    (dict(head_dim=64), "head_dim=128"),
    (dict(num_heads=30), "Q heads must divide"),
    (dict(num_kv_heads=3, num_heads=6, world_size=2, sp_size=2), "Q heads must divide"),
    (dict(max_local_tokens=0), "max_local_tokens"),
    (dict(rank=5, world_size=4, sp_size=4), "rank must be"),
])
def test_constructor_validation(kwargs, match):
    args = dict(rank=0, world_size=2, max_local_tokens=64, sp_size=2)
    args.update(kwargs)
    with pytest.raises(ValueError, match=match):
        FlashUlyssesContext(**args)


def test_layout_properties_match_reference_formulas():
    """base_tp_size, local/output heads and packed width (context.py:95-117)."""
    ctx = object.__new__(FlashUlyssesContext)
    ctx.world_size, ctx.sp_size, ctx.num_heads, ctx.num_kv_heads, ctx.head_dim = 8, 4, 32, 8, 128
    assert ctx.base_tp_size == 2
    assert (ctx.local_q_heads, ctx.local_kv_heads) == (16, 4)
    assert (ctx.output_q_heads, ctx.output_kv_heads) == (4, 1)
    assert ctx.packed_width == 24 * 128


class FakeLib:
    """Records buffer calls; addresses encode (rank, serial)."""

    def __init__(self, rank):
        self.rank = rank
        self.serial = 0
        self.imported, self.closed, self.freed = [], [], []

    def fu_buffer_alloc(self, dev, nbytes, out):
        self.serial += 1
        out._obj.value = (self.rank + 1) << 32 | self.serial << 8
        return 0

    def fu_buffer_export(self, dev, ptr, handle):
        data = f"{ptr:#x}".encode().ljust(64, b"\0")
        ctypes.memmove(handle, data, 64)
        return 0

    def fu_buffer_import(self, dev, handle, out):
        src = int(handle.rstrip(b"\0").decode(), 16)
        self.imported.append(src)
        out._obj.value = src | 1          # "mapped" view of the peer's buffer
        return 0

    def fu_buffer_close(self, dev, ptr):
        self.closed.append(ptr)
        return 0

    def fu_buffer_free(self, dev, ptr):
        self.freed.append(ptr)
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, sp, port, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from flash_ulysses_b200 import _C

        fake = FakeLib(rank)
        _C.lib = fake
        _C.tensor_from_device_ptr = lambda ptr, shape, dtype, device: torch.empty(shape, dtype=dtype)
        start = rank // sp * sp
        peers = list(range(start, start + sp))
        t = _C.ParallelTensor((16, 128), torch.bfloat16, rank, world, False, peers=peers,
                              device=torch.device("cuda", 0))
        assert t.data_.shape == (16, 128)
        assert t.local_rank_ == rank and t.local_world_size_ == world
        for r in peers:
            p = t.peer_ptr(r)
            assert (p >> 32) - 1 == r, (r, hex(p))          # rank r's buffer
            assert (p & 1) == (r != rank)                     # own buffer is not imported
        assert len(fake.imported) == sp - 1
        with pytest.raises(KeyError):
            t.peer_ptr((start + sp) % world if world > sp else -1)
        t.close()
        assert sorted(fake.closed) == sorted(x | 1 for x in fake.imported)
        assert len(fake.freed) == 1
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # pragma: no cover - reported to the parent
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("world,sp", [(2, 2), (4, 2)])
def test_parallel_tensor_exchange_over_gloo(world, sp):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, sp, _free_port(), errq), nprocs=world, join=True,
                       start_method="spawn")
    assert errq.empty()
