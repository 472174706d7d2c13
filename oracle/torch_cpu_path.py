"""The reference's torch CPU path for the shift load, restated.  TEST INFRASTRUCTURE ONLY.

Used as the timed CPU baseline (``bench.py`` cpu_baseline and ``--impl
reference``) and cross-checked bit for bit against :mod:`oracle.shift_oracle`
in the tests.  It follows the pass structure of the reference's
``scatter_shifted_torch`` (acrosley/marathon src/marathon/shift_kernels.py:141-159),
the function the reference dispatches to whenever it has no GPU
(``:180-181``): upcast K to fp32, materialise ``rotate_half``, two broadcast
products and a sum, downcast, concatenate with V, then one advanced-index
scatter into the paged cache, one layer per call as the connector's load loop
and the reference micro-benchmark do (vllm_shift_connector.py:505-518,
scripts/bench_shift_copy.py:41-53).
"""

from __future__ import annotations

import torch


def emb_tables(table: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Broadcast ``emb_cos``/``emb_sin`` of a ``[2, half]`` table (shift_kernels.py:83-84)."""
    c, s = table[0].float(), table[1].float()
    return torch.cat((c, c)), torch.cat((s, s))


def scatter_layer(src, kv, slots, block_size: int, hnd: bool, emb) -> None:
    """One layer: rows ``src[n, heads, 2D]`` into fused paged ``kv`` at ``slots``.

    ``emb`` is ``(emb_cos, emb_sin)`` or None for a plain scatter.
    """
    d = src.shape[-1] // 2
    k = src[..., :d]
    if emb is not None:
        emb_cos, emb_sin = emb
        kf = k.to(torch.float32)
        h = kf.shape[-1] // 2
        turned = torch.cat((-kf[..., h:], kf[..., :h]), dim=-1)
        k = (kf * emb_cos + turned * emb_sin).to(kv.dtype)
    blk = torch.div(slots, block_size, rounding_mode="floor")
    off = slots - blk * block_size
    rows = torch.cat((k, src[..., d:]), dim=-1)
    if hnd:
        kv[blk, :, off] = rows
    else:
        kv[blk, off] = rows


def load_layers(srcs, kvs, slots, block_size: int, hnd: bool, emb) -> None:
    """The connector's per-layer loop over one load."""
    for src, kv in zip(srcs, kvs, strict=True):
        scatter_layer(src, kv, slots, block_size, hnd, emb)


def scatter_layer_e4m3(src, kv, slots, block_size: int, hnd: bool, emb, k_scale: float) -> None:
    """The same layer for e4m3 codes: dequantise with ``k_scale``, rotate, divide by it,
    saturate to +-448, round to e4m3; V codes copied.  ``src``/``kv`` are
    ``torch.float8_e4m3fn`` tensors (the reference has no scale handling; this is
    the requantisation the build defines for FP8 caches).
    """
    d = src.shape[-1] // 2
    k = src[..., :d]
    if emb is not None:
        emb_cos, emb_sin = emb
        kf = k.to(torch.float32) * k_scale
        h = kf.shape[-1] // 2
        turned = torch.cat((-kf[..., h:], kf[..., :h]), dim=-1)
        r = kf * emb_cos + turned * emb_sin
        k = (r / k_scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    blk = torch.div(slots, block_size, rounding_mode="floor")
    off = slots - blk * block_size
    rows = torch.cat((k.view(torch.uint8), src[..., d:].view(torch.uint8)), dim=-1)
    target = kv.view(torch.uint8)
    if hnd:
        target[blk, :, off] = rows
    else:
        target[blk, off] = rows
