"""Ragged, paged restore: page-table gather + dequant + RoPE shift in one launch.

The reference restores a request by gathering its pool blocks on the host
(PinnedKVPool.get_coalesced_views, speccache/cache/pinned_pool.py:392-464), copying
them, and running the key/value kernels per chunk (speccache/cache/engine.py:441-601).
Here the INT8 pool lives on the GPU and one launch gathers every request's pages
through its page table, shifts its keys by its own ``delta_p`` and writes contiguous
caches.

Device-side checks never fault: a bad page id, length or output offset is skipped and
reported through a per-device status word, read with :func:`paged_status`.
"""

from __future__ import annotations

import torch

from .. import _lib
from .staging import host_array, to_device
from .validation import require_cuda

_STATUS: dict[int, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _STATUS.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = w
    return w


def paged_status(device: torch.device | str | int | None = None, reset: bool = True) -> int:
    """Read (and by default clear) the paged kernels' status bits on ``device``.

    Synchronises with the device's current stream.  Bits: SC_STATUS_BAD_PAGE_ID (1),
    SC_STATUS_BAD_SEQ_LEN (2), SC_STATUS_BAD_OUT_OFFSET (4).
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(
        device if not isinstance(device, int) else f"cuda:{device}")
    w = _status_word(dev)
    v = int(w.item())
    if reset:
        w.zero_()
    return v


def restore_paged(
    pool_kq: torch.Tensor | None,
    pool_ks: torch.Tensor | None,
    pool_vq: torch.Tensor | None,
    pool_vs: torch.Tensor | None,
    page_table,
    seq_lens,
    delta_ps,
    *,
    theta: float = 10000.0,
    out_dtype: torch.dtype = torch.bfloat16,
    k_out: torch.Tensor | None = None,
    v_out: torch.Tensor | None = None,
    out_offsets=None,
    delta_p_per_page: bool = False,
    fp32_intermediate: bool = False,
) -> tuple[torch.Tensor | None, torch.Tensor | None, torch.Tensor]:
    """Restore ``R`` ragged requests from a paged INT8 pool.

    Args:
        pool_kq, pool_vq: int8 ``[n_pages, page, H, D]`` (either may be None).
        pool_ks, pool_vs: float16 ``[n_pages, page, H, 1]`` (or ``[n_pages, page, H]``).
        page_table: int32 ``[R, max_pages]`` page ids (host or device).
        seq_lens: ``[R]`` token counts.  Host values are needed to size packed outputs; if
            ``k_out``/``v_out`` and ``out_offsets`` are all given they may live on the device.
        delta_ps: ``[R]`` shifts (or ``[R, max_pages]`` with ``delta_p_per_page``).
        k_out, v_out: outputs; default packed ``[sum(seq_lens), H, D]`` of ``out_dtype``.
        out_offsets: ``[R]`` element offset of each request's first token in the outputs;
            default: packed (cumulative lengths times the token stride).

    Returns ``(k_out, v_out, cu_seqlens)`` with ``cu_seqlens`` int64 ``[R + 1]`` on the host
    (empty when the lengths were given on the device).
    """
    ref = pool_kq if pool_kq is not None else pool_vq
    if ref is None:
        raise ValueError("neither K nor V pool given")
    if ref.ndim != 4 or ref.dtype != torch.int8:
        raise ValueError(f"pools must be int8 [n_pages, page, H, D], got {tuple(ref.shape)} {ref.dtype}")
    require_cuda(ref)
    dev = ref.device
    n_pages, page, h, d = ref.shape
    for q, s in ((pool_kq, pool_ks), (pool_vq, pool_vs)):
        if q is None:
            continue
        if q.shape != ref.shape or q.dtype != torch.int8 or q.device != dev:
            raise ValueError("K and V pools must match in shape, dtype and device")
        if s is None or s.dtype != torch.float16 or s.numel() != n_pages * page * h or not s.is_contiguous():
            raise ValueError("pool scales must be contiguous float16 [n_pages, page, H(, 1)]")
        if not q.is_contiguous():
            raise ValueError("pools must be contiguous")
    table = host_array(page_table, torch.int32)
    if table.ndim != 2:
        raise ValueError(f"page_table must be [R, max_pages], got {tuple(table.shape)}")
    n_req, max_pages = table.shape
    lens_dev = isinstance(seq_lens, torch.Tensor) and seq_lens.is_cuda
    if lens_dev:
        lens_host = None
    else:
        lens_host = torch.as_tensor(seq_lens, dtype=torch.int64).reshape(-1)
        if lens_host.numel() != n_req:
            raise ValueError(f"seq_lens has {lens_host.numel()} entries for {n_req} requests")
        if (lens_host < 0).any() or (lens_host > max_pages * page).any():
            raise ValueError(f"seq_lens must lie in [0, {max_pages * page}]")
    lens = host_array(seq_lens if lens_dev else lens_host, torch.int32)
    dps = host_array(delta_ps, torch.float32)
    expect = n_req * max_pages if delta_p_per_page else n_req
    if dps.numel() != expect:
        raise ValueError(f"delta_ps has {dps.numel()} entries, expected {expect}")
    cu = torch.zeros(n_req + 1, dtype=torch.int64)
    if lens_host is not None:
        cu[1:] = torch.cumsum(lens_host, 0)
    total = int(cu[-1])
    need_alloc = (pool_kq is not None and k_out is None) or (pool_vq is not None and v_out is None)
    if need_alloc and lens_host is None:
        raise ValueError("seq_lens must be on the host when the outputs are allocated here")
    if pool_kq is not None and k_out is None:
        k_out = torch.empty((total, h, d), dtype=out_dtype, device=dev)
    if pool_vq is not None and v_out is None:
        v_out = torch.empty((total, h, d), dtype=k_out.dtype if k_out is not None else out_dtype,
                            device=dev)
    out = k_out if k_out is not None else v_out
    if out.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"outputs must be float16 or bfloat16, got {out.dtype}")
    if k_out is not None and v_out is not None and (
            k_out.stride() != v_out.stride() or k_out.dtype != v_out.dtype or k_out.numel() != v_out.numel()):
        raise ValueError("k_out and v_out must share dtype, size and strides")
    if out.ndim != 3 or out.shape[1:] != (h, d):
        raise ValueError(f"outputs must be [tokens, {h}, {d}] views, got {tuple(out.shape)}")
    if out_offsets is None:
        if lens_host is None:
            raise ValueError("out_offsets are required when seq_lens live on the device")
        offs = cu[:-1] * out.stride(0)
    else:
        offs = host_array(out_offsets, torch.int64)
    if lens_host is not None and total == 0:
        return k_out, v_out, cu
    table, lens, dps, offs = to_device([table, lens, dps, offs], dev)
    status = _status_word(dev)
    flags = _lib.SC_FLAG_FP32_INTERMEDIATE if fp32_intermediate else 0
    # The kernel bounds every write by the extent of the output's storage from its data_ptr.
    numel = min(o.untyped_storage().nbytes() // o.element_size() - o.storage_offset()
                for o in (k_out, v_out) if o is not None)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.sc_restore_paged(
            n_req, max_pages, page, h, d, n_pages,
            _lib.ptr(pool_kq), _lib.ptr(pool_ks), _lib.ptr(pool_vq), _lib.ptr(pool_vs),
            table.data_ptr(), table.stride(0), lens.data_ptr(),
            dps.data_ptr(), 1 if delta_p_per_page else 0, float(theta),
            _lib.inv_freq_ptr(d, theta),
            _lib.ptr(k_out) if pool_kq is not None else None,
            _lib.ptr(v_out) if pool_vq is not None else None,
            offs.data_ptr(), _lib.strides(out.stride(0), out.stride(1), out.stride(2)),
            numel, _lib.DTYPE_CODE[out.dtype], status.data_ptr(), flags,
            _lib.stream_handle(dev))
    _lib.check(rc, "sc_restore_paged")
    return k_out, v_out, (cu if lens_host is not None else torch.empty(0, dtype=torch.int64))
