"""Symmetric device regions shared by the ranks of one node (libclefq clefq_comm_*).

Each rank allocates one region of the same size; the host exchanges CUDA IPC handles once
over torch.distributed, after which the fused entry points (clefq_tp_mlp, clefq_moe_ep_layer)
store into peers' regions over NVLink from inside their kernels and order their phases with
bounded device barriers.  No NCCL call is on those data paths.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def all_gather_rows(out: torch.Tensor, inp: torch.Tensor, group):
    """out[g] = inp of rank g (out has a leading world dimension)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), inp.contiguous(), group=group)


class Comm:
    """This rank's symmetric region, mapped into every rank of `group` (clefq_comm_*).

    Collective: every rank constructs it with the same `region_bytes` (at least what the
    fused entry points it serves ask for: `tp_mlp_region_bytes`, `ep_layer_region_bytes`).
    Without an initialised process group it is a one-rank communicator."""

    def __init__(self, region_bytes: int, group=None, timeout_ms: int | None = None):
        from . import _call, lib
        distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        self.region_bytes = int(region_bytes)
        hb = lib().clefq_comm_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        self._comm = ctypes.c_void_p()
        _call("clefq_comm_create", self.rank, self.world, self.region_bytes, ctypes.byref(self._comm), handle)
        if self.world > 1:
            dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
            mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(dev)
            every = torch.empty((self.world, hb), dtype=torch.uint8, device=dev)
            all_gather_rows(every, mine, group)
            _call("clefq_comm_open", self._comm, ctypes.create_string_buffer(every.cpu().numpy().tobytes()))
        if timeout_ms:
            _call("clefq_comm_set_timeout_ms", self._comm, int(timeout_ms))
        if self.world > 1:
            dist.barrier(group)

    @property
    def handle(self):
        if self._comm is None:
            raise RuntimeError("Comm is closed")
        return self._comm

    def barrier(self):
        from . import _call, _stream
        _call("clefq_comm_barrier", self.handle, _stream())

    def close(self, group=None):
        """Releases the region once every rank's device work on it is done.  Collective for a
        group of more than one rank: no rank frees its region while a peer may still store
        into it or hold it mapped."""
        from . import _call
        if self._comm is not None:
            torch.cuda.synchronize()
            if self.world > 1 and dist.is_initialized():
                dist.barrier(group)
            _call("clefq_comm_destroy", self._comm)
            self._comm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
