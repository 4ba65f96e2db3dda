"""Host side of the tensor-parallel decode (one process per GPU).

The library shards the model itself (``gpt2b_tp_shard_image``) and runs the
collectives with NCCL; the host only has to agree on a group id.  Rank 0
creates the 128-byte NCCL unique id and the ranks share it through
``torch.distributed`` (any backend: gloo on CPU, nccl on GPUs), then each rank
builds its engine with :func:`engine`.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import check, lib
from .engine import WMODES


def plan(cfg: dict, rank: int, size: int) -> dict:
    """This rank's shard: first head and head count, first FC row and FC rows,
    first vocab row and vocab rows (``gpt2b_tp_plan``)."""
    c = (ctypes.c_int * 6)(cfg["maxT"], cfg["V"], cfg["Vp"], cfg["L"], cfg["NH"], cfg["C"])
    out = (ctypes.c_int * 6)()
    check(lib().gpt2b_tp_plan(c, int(rank), int(size), out), "gpt2b_tp_plan")
    h0, nh, f0, fl, v0, vr = list(out)
    return dict(h0=h0, heads=nh, f0=f0, f_rows=fl, v0=v0, v_rows=vr)


def shard_image(image: bytes, scales, wmode: str, rank: int, size: int):
    """This rank's parameter tensors (file order, one byte string) and scale
    array (``gpt2b_tp_shard_image``)."""
    img = np.frombuffer(image, dtype=np.uint8)
    sc_ptr, nsc = None, 0
    if scales is not None:
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        sc_ptr, nsc = scales.ctypes.data_as(ctypes.c_void_p), scales.size
    nb, ns = ctypes.c_size_t(), ctypes.c_size_t()
    args = (img.ctypes.data_as(ctypes.c_void_p), img.size, sc_ptr, nsc, WMODES[wmode], int(rank), int(size))
    check(lib().gpt2b_tp_shard_image(*args, None, ctypes.byref(nb), None, ctypes.byref(ns)), "gpt2b_tp_shard_image")
    out = np.zeros(nb.value, np.uint8)
    osc = np.zeros(max(ns.value, 1), np.float32)
    check(lib().gpt2b_tp_shard_image(*args, out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(nb),
                                     osc.ctypes.data_as(ctypes.c_void_p), ctypes.byref(ns)), "gpt2b_tp_shard_image")
    return out.tobytes(), (osc[: ns.value] if ns.value else None)


def new_group_id() -> bytes:
    """A fresh 128-byte NCCL unique id (``gpt2b_nccl_unique_id``)."""
    buf = ctypes.create_string_buffer(128)
    check(lib().gpt2b_nccl_unique_id(buf), "gpt2b_nccl_unique_id")
    return buf.raw


def shared_group_id(rank: int) -> bytes:
    """Rank 0's new id, broadcast to every rank of the default
    ``torch.distributed`` process group."""
    import torch.distributed as dist
    obj = [new_group_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def all_gather_bytes(data: bytes) -> list:
    """Every rank's ``data`` in rank order, through the default
    ``torch.distributed`` process group."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, data)
    return out


def connect(eng, exchange=all_gather_bytes) -> None:
    """Map every rank's exchange arena into this rank's engine (collective):
    the persistent kernel then runs the group's decode with peer stores over
    NVLink instead of NCCL calls.  ``exchange(bytes) -> list[bytes]`` gathers
    one value per rank in rank order."""
    h = ctypes.create_string_buffer(64)
    check(lib().gpt2b_engine_tp_ipc_handle(eng._h, h), "gpt2b_engine_tp_ipc_handle")
    handles = exchange(h.raw)
    buf = ctypes.create_string_buffer(b"".join(handles), 64 * len(handles))
    check(lib().gpt2b_engine_tp_connect(eng._h, buf, len(handles)), "gpt2b_engine_tp_connect")


def engine(image: bytes, wmode: str, kvmode: str, scales, rank: int, size: int, group_id: bytes,
           p2p: bool = True, exchange=all_gather_bytes):
    """This rank's engine (collective over the group).  With ``p2p`` the ranks'
    exchange arenas are mapped into each other (:func:`connect`) and decoding
    runs in the persistent kernel; otherwise the per-kernel path with NCCL."""
    from .engine import Engine
    eng = Engine.from_buffer_tp(image, wmode, kvmode, scales, rank, size, group_id)
    if p2p and size > 1:
        try:
            connect(eng, exchange)
        except Exception:
            eng.close()
            raise
    return eng
