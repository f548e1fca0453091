"""Gather KV-head shards onto one GPU without a separate collective.

With the restore sharded by KV head (one process per GPU, each restoring its own heads from
its own pinned slab over its own PCIe link), a consumer that is not tensor-parallel needs all
heads on one GPU.  Instead of restoring locally and then running an all-gather, each rank's
restore kernel stores its shard directly into the owner GPU's full cache: the owner exports
the cache (CUDA IPC), the others map it, and their kernels write it with ordinary stores over
NVLink.  The shard lands in the owner's memory as it is restored, layer by layer, overlapped
with the next layer's PCIe copy.

Ordering: the owner may read the caches once every writer's stream has completed (the helper
synchronises its own stream; the caller then runs a barrier, e.g. ``torch.distributed.barrier``).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _lib
from .sharding import head_shard

_NAME_TO_DTYPE = {"float16": torch.float16, "bfloat16": torch.bfloat16}


class SharedBuffer:
    """Device address of another process's buffer, mapped on the current device."""

    def __init__(self, desc: dict) -> None:
        lib = _lib.load()
        handle = ctypes.create_string_buffer(bytes(desc["handle"]), _lib.SC_IPC_HANDLE_BYTES)
        base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(lib.sc_ipc_import(handle, int(desc["offset"]), ctypes.byref(base),
                                     ctypes.byref(ptr)), "sc_ipc_import")
        self._base = base
        self.ptr = int(ptr.value)
        self.shape = tuple(desc["shape"])
        self.stride = tuple(desc["stride"])
        self.dtype = _NAME_TO_DTYPE[desc["dtype"]]
        self.numel = int(desc["numel"])

    @staticmethod
    def describe(t: torch.Tensor) -> dict:
        """Export ``t`` (on the calling process's device) for other processes to map."""
        if not t.is_cuda or t.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError("shared buffers are float16/bfloat16 CUDA tensors")
        lib = _lib.load()
        handle = ctypes.create_string_buffer(_lib.SC_IPC_HANDLE_BYTES)
        offset = ctypes.c_int64(0)
        _lib.check(lib.sc_ipc_export(ctypes.c_void_p(t.data_ptr()), handle, ctypes.byref(offset)),
                   "sc_ipc_export")
        return {"handle": bytes(handle.raw), "offset": int(offset.value), "shape": list(t.shape),
                "stride": list(t.stride()), "dtype": str(t.dtype).replace("torch.", ""),
                "numel": t.untyped_storage().nbytes() // t.element_size() - t.storage_offset()}

    def close(self) -> None:
        if self._base is not None and self._base.value:
            _lib.load().sc_ipc_close(self._base)
            self._base = None


class HeadShardGather:
    """Restore this rank's KV-head shard straight into the owner rank's full caches.

    Args:
        pipeline: this rank's ``KVRestorePipeline`` (its slabs hold the rank's heads).
        k_full, v_full: on the owner, the ``[L, T, H_total, D]`` caches (contiguous per token:
            strides ``[T*H*D, H*D, D, 1]``); ``None`` on the other ranks.
        owner, rank, world_size: ranks of the gather; ``num_kv_heads`` is ``H_total``.
        group: process group used once to exchange the IPC handles.
    """

    def __init__(self, pipeline, k_full: torch.Tensor | None, v_full: torch.Tensor | None, *,
                 owner: int, rank: int, world_size: int, num_kv_heads: int, group=None) -> None:
        import torch.distributed as dist

        self.pipeline, self.rank, self.owner = pipeline, rank, owner
        sl = head_shard(num_kv_heads, world_size, rank)
        if sl.stop - sl.start != pipeline.num_kv_heads:
            raise ValueError(f"pipeline holds {pipeline.num_kv_heads} heads, shard is {sl}")
        descs = [None, None]
        if rank == owner:
            for x in (k_full, v_full):
                if x is None or x.ndim != 4 or x.shape[2] != num_kv_heads or x.stride(3) != 1:
                    raise ValueError("owner caches must be [L, T, H, D] with unit dim stride")
            descs = [SharedBuffer.describe(k_full), SharedBuffer.describe(v_full)]
        if world_size > 1:
            dist.broadcast_object_list(descs, src=owner, group=group)
        self._mapped: list[SharedBuffer] = []
        if rank == owner:
            bases = [(k_full.data_ptr(), descs[0]), (v_full.data_ptr(), descs[1])]
        else:
            self._mapped = [SharedBuffer(d) for d in descs]
            bases = [(m.ptr, d) for m, d in zip(self._mapped, descs)]
        (kb, kd), (vb, vd) = bases
        self.dtype = _NAME_TO_DTYPE[kd["dtype"]]
        item = torch.empty((), dtype=self.dtype).element_size()
        st = kd["stride"]
        if list(vd["stride"]) != list(st) or vd["shape"] != kd["shape"]:
            raise ValueError("K and V caches must share shape and strides")
        layers = pipeline.num_layers
        self.out_strides = (st[1], st[2], 1)
        first = sl.start * st[2]
        self.k_ptrs = [kb + (layer * st[0] + first) * item for layer in range(layers)]
        self.v_ptrs = [vb + (layer * st[0] + first) * item for layer in range(layers)]
        # elements the kernel may touch from the last layer's pointer (the tightest bound)
        self.out_numel = min(kd["numel"], vd["numel"]) - ((layers - 1) * st[0] + first)

    def restore(self, block_ids, delta_ps, *, theta: float = 10000.0) -> None:
        """Enqueue the restore of this rank's shard into the owner's caches."""
        self.pipeline.restore_into(block_ids, delta_ps, self.k_ptrs, self.v_ptrs, self.out_strides,
                                   self.out_numel, self.dtype, theta=theta)

    def close(self) -> None:
        for m in self._mapped:
            m.close()
        self._mapped = []
