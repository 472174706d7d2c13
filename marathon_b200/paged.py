"""Describe vLLM paged KV caches to the native kernels: base pointers plus strides.

A paged cache layer is reduced to a K base, a V base and three element strides
(block, in-block offset, head); the innermost head dimension must be
contiguous.  That one description covers every layout the shift path meets:

``nhd``    fused ``[blocks, block_size, heads, 2*head_size]`` (vLLM's default
           fused layout, the reference connector's NHD case,
           ``src/marathon/vllm_shift_connector.py:397-401``)
``hnd``    fused ``[blocks, heads, block_size, 2*head_size]``
``split``  ``(2, blocks, block_size, heads, head_size)``: vLLM 0.22's
           FlashAttention backend, K = ``kv[0]``, V = ``kv[1]``; any physical
           stride order vLLM picks is read off the tensor's strides
``split_blocks``  ``(blocks, 2, block_size, heads, head_size)``: FlashInfer

Layout detection for 4-D tensors follows the reference exactly
(``vllm_shift_connector.py:399-401``): HND iff ``shape[2] == block_size`` and
``shape[1] != block_size``; when both equal the block size it is NHD.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

_DTYPES = {
    torch.bfloat16: _lib.BF16,
    torch.float16: _lib.F16,
    torch.float32: _lib.F32,
    torch.float8_e4m3fn: _lib.E4M3,
}


def dtype_code(dtype: torch.dtype, fp8: bool = False) -> int:
    """Native dtype code of a cache tensor; ``uint8`` means e4m3 when ``fp8``."""
    if dtype == torch.uint8 and fp8:
        return _lib.E4M3
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise _lib.ShiftError(f"unsupported KV cache dtype {dtype}") from None


def paged_strides(kv: torch.Tensor, hnd: bool) -> tuple[int, int, int]:
    """(block, head, in-block-offset) strides of a fused 4-D paged KV tensor.

    Same contract as the reference's ``_paged_strides``
    (``src/marathon/shift_kernels.py:135-138``).
    """
    s = kv.stride()
    return (s[0], s[1], s[2]) if hnd else (s[0], s[2], s[1])


def detect_hnd(shape: tuple[int, ...], block_size: int) -> bool:
    """The reference's 4-D layout rule (``vllm_shift_connector.py:399-401``)."""
    hnd = shape[2] == block_size and shape[1] != block_size
    if shape[1] == block_size and shape[2] == block_size:
        hnd = False
    return hnd


@dataclass(frozen=True)
class PagedLayout:
    """Geometry shared by every layer of a paged cache (element strides)."""

    kind: str
    num_blocks: int
    block_size: int
    heads: int
    head_size: int
    blk_stride: int
    off_stride: int
    head_stride: int
    dtype: int  # native dtype code
    elem_bytes: int
    v_offset: int  # elements from a layer's K base to its V base

    def struct(self) -> _lib.Paged:
        return _lib.Paged(
            self.blk_stride,
            self.off_stride,
            self.head_stride,
            self.num_blocks,
            self.block_size,
            self.heads,
            self.head_size,
            self.dtype,
        )

    @property
    def num_slots(self) -> int:
        return self.num_blocks * self.block_size


def describe(
    kv: torch.Tensor,
    block_size: int,
    layout: str | None = None,
    hnd: bool | None = None,
    fp8: bool = False,
) -> PagedLayout:
    """Describe one layer's cache tensor. ``layout`` overrides detection."""
    shape = tuple(kv.shape)
    es = kv.element_size()
    code = dtype_code(kv.dtype, fp8)
    if layout is None:
        if kv.dim() == 4:
            layout = "hnd" if (hnd if hnd is not None else detect_hnd(shape, block_size)) else "nhd"
        elif kv.dim() == 5:
            layout = "split" if shape[0] == 2 else "split_blocks"
        else:
            raise _lib.ShiftError(f"expected a 4-D fused or 5-D split KV cache, got {shape}")
    s = kv.stride()
    if layout in ("nhd", "hnd"):
        if kv.dim() != 4 or shape[3] % 2:
            raise _lib.ShiftError(f"fused layout needs [blocks, ., ., 2*head_size], got {shape}")
        head_size = shape[3] // 2
        blk, head, off = paged_strides(kv, layout == "hnd")
        heads = shape[1] if layout == "hnd" else shape[2]
        bs = shape[2] if layout == "hnd" else shape[1]
        inner = s[3]
        v_offset = head_size
        num_blocks = shape[0]
    elif layout == "split":
        if kv.dim() != 5 or shape[0] != 2:
            raise _lib.ShiftError(f"split layout needs (2, blocks, bs, heads, D), got {shape}")
        num_blocks, bs, heads, head_size = shape[1:]
        blk, off, head, inner = s[1], s[2], s[3], s[4]
        v_offset = s[0]
    elif layout == "split_blocks":
        if kv.dim() != 5 or shape[1] != 2:
            raise _lib.ShiftError(f"split_blocks layout needs (blocks, 2, bs, heads, D), got {shape}")
        num_blocks, _, bs, heads, head_size = shape
        blk, off, head, inner = s[0], s[2], s[3], s[4]
        v_offset = s[1]
    else:
        raise _lib.ShiftError(f"unknown paged layout {layout!r}")
    if bs != block_size:
        raise _lib.ShiftError(f"cache block size {bs} != block_size {block_size}")
    if inner != 1:
        raise _lib.ShiftError("the head dimension of the KV cache must be contiguous")
    return PagedLayout(
        kind=layout,
        num_blocks=int(num_blocks),
        block_size=int(block_size),
        heads=int(heads),
        head_size=int(head_size),
        blk_stride=int(blk),
        off_stride=int(off),
        head_stride=int(head),
        dtype=code,
        elem_bytes=es,
        v_offset=int(v_offset),
    )


def base_pointers(kv: torch.Tensor, geo: PagedLayout) -> tuple[int, int]:
    """(K base, V base) device addresses of one layer."""
    k = kv.data_ptr()
    return k, k + geo.v_offset * geo.elem_bytes


class KVLayers:
    """The registered paged caches of all layers: one geometry, per-layer bases.

    Built once when vLLM registers its caches (the reference does its layout
    detection at the same point, ``vllm_shift_connector.py:393-412``).  Holds
    the per-layer K/V base pointers on the device for the batched kernels.
    """

    def __init__(
        self,
        caches: dict[str, torch.Tensor] | list[torch.Tensor],
        block_size: int,
        layout: str | None = None,
        hnd: bool | None = None,
        fp8: bool = False,
    ) -> None:
        items = list(caches.items()) if isinstance(caches, dict) else list(enumerate(caches))
        if not items:
            raise _lib.ShiftError("no KV cache layers to register")
        self.names = [name for name, _ in items]
        self.tensors = [t for _, t in items]
        first = self.tensors[0]
        self.geometry = describe(first, block_size, layout, hnd, fp8)
        for name, t in items[1:]:
            g = describe(t, block_size, self.geometry.kind, fp8=fp8)
            if g != self.geometry:
                raise _lib.ShiftError(f"layer {name!r} has a different cache geometry")
        self.device = first.device
        ptrs = [base_pointers(t, self.geometry) for t in self.tensors]
        self.k_host = [k for k, _ in ptrs]
        self.v_host = [v for _, v in ptrs]
        if first.is_cuda:
            both = torch.tensor(self.k_host + self.v_host, dtype=torch.int64)
            dev = both.to(self.device)
            self.k_ptrs = dev[: len(ptrs)]
            self.v_ptrs = dev[len(ptrs) :]
        else:
            self.k_ptrs = self.v_ptrs = None
        self.index = {name: i for i, name in enumerate(self.names)}

    def __len__(self) -> int:
        return len(self.names)
