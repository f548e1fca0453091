"""Pinned-host -> GPU multi-layer KV restore pipeline (C++ in ``libspeccache_b200.so``).

Python face of ``sc_pipeline_*``: it owns pinned host slabs laid out like the
reference's unified multi-layer slabs (speccache/serving/kv_injector.py:171-192,
``[L, blocks, chunk, H, D]`` int8 and ``[L, blocks, chunk, H, 1]`` fp16), and restores a
list of blocks for every layer: per stage of the block list (or per layer), H2D copies (one
per run of consecutive block ids, every layer in one copy) on its own transfer stream into a
ring of device slots, joined by events to the restore kernel on the caller's current stream,
so the next stage's copy overlaps this stage's kernel.  This replaces the Python loops of
``MultiLayerKVInjector.reconstruct_and_inject_multi_layer`` (kv_injector.py:392-498)
and ``SpecCacheEngine.execute_async_dma_and_rope`` (speccache/cache/engine.py:441-601).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _lib


def _host_view(addr: int, shape: tuple[int, ...], np_dtype, torch_dtype=None) -> torch.Tensor:
    n = int(np.prod(shape))
    ctype = {np.int8: ctypes.c_int8, np.int16: ctypes.c_int16}[np_dtype]
    arr = np.ctypeslib.as_array((ctype * n).from_address(addr)).reshape(shape)
    t = torch.from_numpy(arr)
    return t.view(torch_dtype) if torch_dtype is not None else t


class KVRestorePipeline:
    """Multi-layer restore from pinned host slabs into per-layer GPU caches.

    Args:
        num_layers, num_blocks, chunk_size, num_kv_heads, head_dim: slab geometry.
        device: CUDA device of the restore.
        max_restore_blocks: most blocks one restore may ask for (sizes the device slots);
            default ``num_blocks``.
        n_slots: device staging slots (2 = double buffering).
        numa_local: allocate the slabs from a thread bound to the GPU's NUMA node.
        write_combined: pin the slabs write-combined (host writes and GPU reads only; host
            reads of the slab views become very slow).
        per_layer: always restore layer by layer.  By default a restore goes in stages of
            its block list (up to 64 MiB of K and V codes over all layers each, the last stage
            one block): per stage one 3-D copy per run of consecutive block ids and one launch
            for every layer, so a scattered block list costs one copy per run; a restore of
            fewer than 8 blocks that fits one stage is one launch.
        split_kv_copies: move a run's K and V codes as two 2-D copies instead of one 3-D copy
            (what a slab beyond the device's 2 GB copy pitch does anyway); for comparisons and
            tests.
    """

    def __init__(self, num_layers: int, num_blocks: int, chunk_size: int, num_kv_heads: int,
                 head_dim: int, *, device: torch.device | str | int | None = None,
                 max_restore_blocks: int | None = None, n_slots: int = 2,
                 numa_local: bool = True, write_combined: bool = False,
                 per_layer: bool = False, split_kv_copies: bool = False) -> None:
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        if device.type != "cuda":
            raise RuntimeError(f"KVRestorePipeline needs a CUDA device, got {device}")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.num_layers, self.num_blocks = int(num_layers), int(num_blocks)
        self.chunk_size, self.num_kv_heads, self.head_dim = int(chunk_size), int(num_kv_heads), int(head_dim)
        self.max_restore_blocks = int(max_restore_blocks or num_blocks)
        self._lib = _lib.load()
        self._ptr_arrays: dict[tuple, ctypes.Array] = {}
        handle = ctypes.c_void_p()
        flags = (_lib.SC_PIPE_NUMA_LOCAL if numa_local else 0) | (
            _lib.SC_PIPE_WRITE_COMBINED if write_combined else 0) | (
            _lib.SC_PIPE_PER_LAYER if per_layer else 0) | (
            _lib.SC_PIPE_SPLIT_KV_COPIES if split_kv_copies else 0)
        rc = self._lib.sc_pipeline_create(device.index, self.num_layers, self.num_blocks,
                                          self.chunk_size, self.num_kv_heads, self.head_dim,
                                          self.max_restore_blocks, int(n_slots), flags,
                                          ctypes.byref(handle))
        _lib.check(rc, "sc_pipeline_create")
        self._h = handle
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        _lib.check(self._lib.sc_pipeline_host_slabs(self._h, *[ctypes.byref(p) for p in ptrs]),
                   "sc_pipeline_host_slabs")
        codes = (self.num_layers, self.num_blocks, self.chunk_size, self.num_kv_heads, self.head_dim)
        scales = codes[:4] + (1,)
        self.k_quant = _host_view(ptrs[0].value, codes, np.int8)
        self.k_scale = _host_view(ptrs[1].value, scales, np.int16, torch.float16)
        self.v_quant = _host_view(ptrs[2].value, codes, np.int8)
        self.v_scale = _host_view(ptrs[3].value, scales, np.int16, torch.float16)

    # -- host slab access ---------------------------------------------------------------
    def write_block(self, layer: int, block_id: int, k_quant: torch.Tensor, k_scale: torch.Tensor,
                    v_quant: torch.Tensor, v_scale: torch.Tensor) -> None:
        """Copy one quantised chunk ``[chunk, H, D]`` / ``[chunk, H, 1]`` into the slabs."""
        self.k_quant[layer, block_id].copy_(k_quant)
        self.k_scale[layer, block_id].copy_(k_scale)
        self.v_quant[layer, block_id].copy_(v_quant)
        self.v_scale[layer, block_id].copy_(v_scale)

    # -- restore --------------------------------------------------------------------------
    def restore(self, block_ids, delta_ps, k_out, v_out, *, theta: float = 10000.0) -> None:
        """Enqueue the restore of ``block_ids`` (block i shifted by ``delta_ps[i]``) for
        every layer.  ``k_out`` / ``v_out``: a list of ``num_layers`` ``[n*chunk, H, D]``
        fp16/bf16 views (any token/head strides, unit dim stride) sharing one layout, or one
        ``[num_layers, n*chunk, H, D]`` tensor.  The kernels write only inside these views.
        Completion is ordered on the current CUDA stream; the call does not wait for the
        device unless four earlier restores are still queued behind unfinished kernels."""
        ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32).reshape(-1))
        dps = np.ascontiguousarray(np.asarray(delta_ps, dtype=np.int64).reshape(-1))
        if ids.size != dps.size:
            raise ValueError(f"{ids.size} block ids but {dps.size} shifts")
        dps32 = dps.astype(np.int32)
        if (dps32 != dps).any():
            raise ValueError("shifts must fit in int32")
        shape = (ids.size * self.chunk_size, self.num_kv_heads, self.head_dim)
        kp, kst, dtype = self._layer_pointers(k_out, shape)
        vp, vst, vdt = self._layer_pointers(v_out, shape)
        if vst != kst or vdt != dtype:
            raise ValueError("K and V outputs must share dtype and layout")
        # elements from a layer's address to the end of its view (the kernels' write bound)
        extent = (shape[0] - 1) * kst[0] + (shape[1] - 1) * kst[1] + shape[2]
        self._restore(ids, dps32, kp, vp, kst, extent, dtype, theta)

    def _layer_pointers(self, out, shape):
        """Per-layer output addresses, the common [token, head, dim] strides and the dtype."""
        bad = ValueError(f"outputs must be {self.num_layers} [{shape[0]}, {shape[1]}, {shape[2]}] "
                         f"float16/bfloat16 views on {self.device} sharing one layout (unit dim "
                         "stride), or one tensor with a leading layer dimension")
        dev = self.device.index
        if isinstance(out, torch.Tensor):  # [L, T, H, D]: checked once
            if (out.ndim != 4 or tuple(out.shape) != (self.num_layers,) + shape
                    or out.get_device() != dev or out.stride(3) != 1
                    or out.dtype not in (torch.float16, torch.bfloat16)):
                raise bad
            base, step = out.data_ptr(), out.stride(0) * out.element_size()
            return (tuple([base + layer * step for layer in range(self.num_layers)]),
                    tuple(out.stride()[1:]), out.dtype)
        if len(out) != self.num_layers:
            raise bad
        ref = out[0]
        dtype, st = ref.dtype, ref.stride()
        if dtype not in (torch.float16, torch.bfloat16) or st[2] != 1:
            raise bad
        ptrs = []
        for o in out:
            if o.dtype is not dtype or o.shape != shape or o.stride() != st or o.get_device() != dev:
                raise bad
            ptrs.append(o.data_ptr())
        return tuple(ptrs), st, dtype

    def restore_into(self, block_ids, delta_ps, k_ptrs: list[int], v_ptrs: list[int],
                     out_strides: tuple[int, int, int], out_numel: int,
                     out_dtype: torch.dtype, *, theta: float = 10000.0) -> None:
        """:meth:`restore` into raw device addresses (e.g. another GPU's buffer mapped with
        :class:`~speccache_b200.cache.peer.SharedBuffer`): layer l's token i, head h goes to
        ``k_ptrs[l] + (i * out_strides[0] + h * out_strides[1] + d) * itemsize``; the kernel
        refuses to write beyond ``out_numel`` elements from each pointer."""
        ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32).reshape(-1))
        dps = np.ascontiguousarray(np.asarray(delta_ps, dtype=np.int64).reshape(-1))
        if ids.size != dps.size:
            raise ValueError(f"{ids.size} block ids but {dps.size} shifts")
        if len(k_ptrs) != self.num_layers or len(v_ptrs) != self.num_layers:
            raise ValueError(f"need {self.num_layers} K and V pointers")
        self._restore(ids, dps.astype(np.int32), tuple(map(int, k_ptrs)), tuple(map(int, v_ptrs)),
                      tuple(out_strides), int(out_numel), out_dtype, theta)

    def _restore(self, ids, dps32, k_ptrs, v_ptrs, strides, numel, dtype, theta) -> None:
        if dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"outputs must be float16 or bfloat16, got {dtype}")
        kp, vp = self._pointer_array(k_ptrs), self._pointer_array(v_ptrs)
        rc = self._lib.sc_pipeline_restore(
            self._h, ids.ctypes.data, dps32.ctypes.data, int(ids.size), float(theta),
            _lib.inv_freq_ptr(self.head_dim, theta), kp, vp, _lib.strides(*strides), numel,
            _lib.DTYPE_CODE[dtype], _lib.stream_handle(self.device))
        _lib.check(rc, "sc_pipeline_restore")

    def _pointer_array(self, ptrs: tuple):
        """The per-layer address array for the C call, kept for outputs seen before (a
        serving loop restores into the same cache buffers again and again)."""
        arr = self._ptr_arrays.get(ptrs)
        if arr is None:
            if len(self._ptr_arrays) >= 64:
                self._ptr_arrays.clear()
            arr = self._ptr_arrays[ptrs] = (ctypes.c_void_p * self.num_layers)(*ptrs)
        return arr

    def offload(self, layer: int, block_ids, k: torch.Tensor, v: torch.Tensor) -> None:
        """Enqueue quantize-on-GPU + D2H of freshly computed K/V into the slabs (copies for
        consecutive block ids, one scatter kernel into the mapped slabs for a scattered list).

        ``k`` / ``v``: ``[n * chunk, H, D]`` fp16/bf16/fp32 CUDA tensors; block i's tokens go
        to slab block ``block_ids[i]`` of ``layer``.  The quantisation is bit-exact with the
        reference's ``quantize_kv_int8``.  Ordered before later restores (same transfer
        stream); the host may read the slabs after :meth:`synchronize`.
        """
        ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32).reshape(-1))
        n_tok = ids.size * self.chunk_size
        for x in (k, v):
            if x.shape != (n_tok, self.num_kv_heads, self.head_dim) or x.device != self.device:
                raise ValueError(f"K/V must be [{n_tok}, {self.num_kv_heads}, {self.head_dim}] "
                                 f"on {self.device}, got {tuple(x.shape)} on {x.device}")
            if x.dtype not in _lib.DTYPE_CODE:
                raise TypeError(f"K/V must be float16, bfloat16 or float32, got {x.dtype}")
        if k.dtype != v.dtype:
            raise TypeError("K and V must share a dtype")
        rc = self._lib.sc_pipeline_offload(
            self._h, int(layer), ids.ctypes.data, int(ids.size), k.data_ptr(),
            _lib.strides(*k.stride()), v.data_ptr(), _lib.strides(*v.stride()),
            _lib.DTYPE_CODE[k.dtype], _lib.stream_handle(self.device))
        _lib.check(rc, "sc_pipeline_offload")

    def synchronize(self, timeout: float = 60.0) -> None:
        """Wait for the last restore and offload, polling; raises TimeoutError after
        ``timeout`` seconds."""
        _lib.check(self._lib.sc_pipeline_synchronize(self._h, float(timeout)), "sc_pipeline_synchronize")

    def join(self, stream: torch.cuda.Stream | None = None) -> None:
        """Make ``stream`` (default: the current stream) wait on the GPU for the restores and
        offloads enqueued so far, copies included; the host does not wait."""
        handle = stream.cuda_stream if stream is not None else _lib.stream_handle(self.device)
        _lib.check(self._lib.sc_pipeline_join(self._h, handle), "sc_pipeline_join")

    def restore_launches(self, n_blocks: int) -> int:
        """Kernel launches a restore of ``n_blocks`` blocks issues: one per block stage (1
        below 8 blocks when they fit one stage), one per layer with ``per_layer``."""
        count = ctypes.c_int32(0)
        _lib.check(self._lib.sc_pipeline_restore_launches(self._h, int(n_blocks), ctypes.byref(count)),
                   "sc_pipeline_restore_launches")
        return int(count.value)

    def restore_plan(self, block_ids) -> tuple[int, int]:
        """(kernel launches, copy commands) a restore of ``block_ids`` enqueues: one launch per
        block stage plus the scale gather of a list in several runs; one copy per run of
        consecutive ids within a stage, the scales' copies and the metadata upload."""
        return self._plan(0, block_ids)

    def offload_plan(self, block_ids) -> tuple[int, int]:
        """(kernel launches, copy commands) an offload of one layer into ``block_ids``
        enqueues: the K and V quantize, plus the scatter kernels of a list in several runs
        (else two copies per run)."""
        return self._plan(1, block_ids)

    def _plan(self, offload: int, block_ids) -> tuple[int, int]:
        ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32).reshape(-1))
        launches, copies = ctypes.c_int32(0), ctypes.c_int32(0)
        _lib.check(self._lib.sc_pipeline_plan(self._h, offload, ids.ctypes.data, int(ids.size),
                                              ctypes.byref(launches), ctypes.byref(copies)),
                   "sc_pipeline_plan")
        return int(launches.value), int(copies.value)

    def status(self) -> int:
        """Device status bits of the restore kernels (0 = clean); reading clears them."""
        bits = ctypes.c_int32(0)
        rc = self._lib.sc_pipeline_status(self._h, ctypes.byref(bits))
        if rc not in (_lib.SC_OK, _lib.SC_ERR_OUT_OF_RANGE):
            _lib.check(rc, "sc_pipeline_status")
        return int(bits.value)

    def close(self) -> None:
        """Release the slabs and device buffers; the slab views become unusable."""
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.k_quant = self.k_scale = self.v_quant = self.v_scale = None
            self._lib.sc_pipeline_destroy(h)
            self._h = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self) -> "KVRestorePipeline":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
