"""Generate the golden vectors of the shift path by running the reference itself.

Run once on a machine that has the reference checkout (acrosley/marathon);
the output ``shift_golden.npz`` is committed, so neither the tests nor the GPU
box need the reference at run time:

    MARATHON_REFERENCE=/path/to/marathon/src python tests/golden/make_golden.py

What is recorded (all produced by the reference's own functions on CPU):

* ``inv_freq_*``     the connector's inverse-frequency expression
                     (vllm_shift_connector.py:196-198) for rotary 128/64, theta 1e6/1e4
* ``tab_<d>_*``      ``rope_shift(d, 128, inv, "cpu")`` fields (shift_kernels.py:68-84)
                     plus the fp32 angle ``float(d) * inv_freq``
* ``bf16_src`` / ``bf16_k_<d>``  ``scatter_shifted_torch`` on bf16 rows (the torch
                     path, shift_kernels.py:141-159) at the geometry of
                     tests/test_shift_kernels.py:46-78 (8 heads, 128 dim, block 16,
                     a scattered block table, the run starting mid-block)
* ``f32r_k_<d>``     the same call on fp32 copies of those rows and an fp32 cache:
                     the reference's rotation computed in fp32, before any rounding
                     to the cache dtype (the value the 1-ulp bar is measured from)
* ``f32_digest_*``   sha256 of the fp32 rows ``scatter_shifted`` lands at the Qwen3
                     geometry of tests/test_shift_kernels.py:93-134, both layouts
* ``slots_*``        ``shift_store.slots`` incl. the known answer [30, 31, 12, 13]
                     of tests/test_shift_store.py:24-27
* ``round_*``        torch's fp32 -> bf16 / fp16 / float8_e4m3fn rounding of edge values
* ``hf_*``           keys RoPE'd by transformers' Qwen3RotaryEmbedding at p and
                     p + delta (the identity tests/test_kvshift.py:48-55 pins)
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "shift_golden.npz"
DELTAS_TABLE = [-3000, -1133, -566, -512, -40, -17, -4, -1, 0, 1, 4, 12, 17, 37, 180, 186, 215,
                512, 566, 6759, 10000]
DELTAS_BF16 = [-3000, -4, 0, 4, 186, 10000]
DELTAS_F32 = [0, 1, -1, 17, -17, 566, -566, -1133, 6759]


def _ref():
    src = os.environ.get("MARATHON_REFERENCE")
    if not src:
        sys.exit("set MARATHON_REFERENCE to the reference checkout's src/ directory")
    sys.path.insert(0, src)
    from marathon import shift_kernels, shift_store  # noqa: PLC0415
    from marathon.kvshift import rerotate_keys  # noqa: PLC0415

    return shift_kernels, shift_store, rerotate_keys


def _inv(rotary: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, rotary, 2, dtype=torch.float32) / rotary))


def main() -> None:
    sk, ss, rerotate_keys = _ref()
    out: dict[str, np.ndarray] = {}

    for rot in (128, 64):
        for theta in (1e6, 1e4):
            out[f"inv_freq_{rot}_{int(theta)}"] = _inv(rot, theta).numpy()
    inv = _inv(128, 1e6)

    # --- rotation tables
    out["table_deltas"] = np.asarray(DELTAS_TABLE, dtype=np.int64)
    for d in DELTAS_TABLE:
        sh = sk.rope_shift(d, 128, inv, "cpu")
        out[f"tab_{d}_ang"] = (float(d) * inv).numpy()
        out[f"tab_{d}_cos"] = sh.cos.numpy()
        out[f"tab_{d}_sgn"] = sh.sgn.numpy()
        out[f"tab_{d}_partner"] = sh.partner.numpy()
        out[f"tab_{d}_emb_cos"] = sh.emb_cos.numpy()
        out[f"tab_{d}_emb_sin"] = sh.emb_sin.numpy()
    # partial rotary: head 256, 64 rotating dims
    inv64 = _inv(64, 1e6)
    sh = sk.rope_shift(37, 256, inv64, "cpu")
    out["partial_cos"], out["partial_sgn"] = sh.cos.numpy(), sh.sgn.numpy()
    out["partial_partner"] = sh.partner.numpy()

    # --- bf16 scatter through the torch path
    heads, d, bs, nblocks, n = 8, 128, 16, 64, 40
    g = torch.Generator().manual_seed(20261201)
    src = torch.randn(n, heads, 2 * d, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblocks, generator=g)[: -(-(n + 3) // bs) + 1]
    pos = torch.arange(3, 3 + n)
    slots = table[pos // bs] * bs + pos % bs
    out["bf16_src"] = src.view(torch.int16).numpy().view(np.uint16)
    out["bf16_slots"] = slots.numpy()
    out["bf16_deltas"] = np.asarray(DELTAS_BF16, dtype=np.int64)
    for delta in DELTAS_BF16:
        for hnd in (True, False):
            shape = (nblocks, heads, bs, 2 * d) if hnd else (nblocks, bs, heads, 2 * d)
            kv = torch.zeros(shape, dtype=torch.bfloat16)
            sk.scatter_shifted_torch(src, kv, slots, bs, hnd, sk.rope_shift(delta, d, inv, "cpu"))
            blk, off = slots // bs, slots % bs
            got = kv[blk, :, off] if hnd else kv[blk, off]
            bits = got.view(torch.int16).numpy().view(np.uint16)
            if hnd:
                out[f"bf16_k_{delta}"] = bits[..., :d].copy()
                assert np.array_equal(bits[..., d:], out["bf16_src"][..., d:])
            else:
                assert np.array_equal(bits[..., :d], out[f"bf16_k_{delta}"]), "layout changed values"
            if not hnd:
                # the unrounded value r: the same torch path on fp32 copies of
                # the inputs, so the rotation's result is never cast to bf16
                kv32 = torch.zeros(shape, dtype=torch.float32)
                sk.scatter_shifted_torch(src.float(), kv32, slots, bs, hnd,
                                         sk.rope_shift(delta, d, inv, "cpu"))
                out[f"f32r_k_{delta}"] = kv32[blk, off][..., :d].numpy().copy()
            # everything not in `slots` must still be zero
            mask = torch.ones(nblocks * bs, dtype=torch.bool)
            mask[slots] = False
            rest = kv.permute(0, 2, 1, 3) if hnd else kv
            assert not rest.reshape(nblocks * bs, heads, 2 * d)[mask].any()

    # --- fp32 Qwen3 geometry through the public scatter_shifted (CPU -> torch path)
    src32 = src.to(torch.float32)
    blocks = 12
    g2 = torch.Generator().manual_seed(7)
    slots32 = torch.randperm(blocks * bs, generator=g2)[:n].to(torch.int64)
    out["f32_slots"] = slots32.numpy()
    for delta in DELTAS_F32:
        for hnd in (True, False):
            shape = (blocks, heads, bs, 2 * d) if hnd else (blocks, bs, heads, 2 * d)
            kv = torch.zeros(shape, dtype=torch.float32)
            sk.scatter_shifted(src32, kv, slots32, bs, hnd, sk.rope_shift(delta, d, inv, "cpu"))
            blk, off = slots32 // bs, slots32 % bs
            got = kv[blk, :, off] if hnd else kv[blk, off]
            want = torch.cat((rerotate_keys(src32[..., :d], delta, inv), src32[..., d:]), -1)
            assert torch.allclose(got, want, atol=1e-4)
            tag = f"{delta}_{'hnd' if hnd else 'nhd'}"
            out[f"f32_digest_{tag}"] = np.frombuffer(
                hashlib.sha256(got.contiguous().numpy().tobytes()).digest(), dtype=np.uint8
            )

    # --- slot mapping
    out["slots_known"] = ss.slots([7, 3], 2, 6, block_size=4).numpy()
    g3 = torch.Generator().manual_seed(11)
    bt = torch.randperm(500, generator=g3)[:300].tolist()
    out["slots_bt"] = np.asarray(bt, dtype=np.int64)
    out["slots_bt_out"] = ss.slots(bt, 1061, 4133, 16).numpy()

    # --- rounding of edge values by torch
    edge = torch.tensor(
        [0.0, -0.0, 1.0, -1.0, 1.00390625, 1.01171875, 1.0078125, 3.3895314e38, 3.4e38,
         float("inf"), -float("inf"), 1e-40, -1e-40, 9.2e-41, 5.877472e-39, 65504.0, 65520.0,
         6.1e-5, 5.96e-8, 2.98e-8, 448.0, 464.0, 447.99, 0.001953125, 0.0009765625, 0.00146484375,
         0.0029296875, 240.0, 248.0, 232.0, 17.0, 18.0, 19.0, -17.0, -19.0, 0.1, -0.1, 3.14159],
        dtype=torch.float32,
    )
    rnd = torch.randn(4096, generator=torch.Generator().manual_seed(5)) * 30
    vals = torch.cat((edge, rnd))
    out["round_in"] = vals.numpy()
    out["round_bf16"] = vals.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    out["round_f16"] = vals.to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    clamped = vals.clamp(-448.0, 448.0)
    finite = torch.isfinite(vals)
    out["round_e4m3_in"] = clamped[finite].numpy()
    out["round_e4m3"] = clamped[finite].to(torch.float8_e4m3fn).view(torch.uint8).numpy()

    # --- transformers' Qwen3 rotary: rerotate(K@p, delta) == K@(p+delta)
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config  # noqa: PLC0415
    from transformers.models.qwen3.modeling_qwen3 import (  # noqa: PLC0415
        Qwen3RotaryEmbedding,
        rotate_half,
    )

    cfg = Qwen3Config(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, num_hidden_layers=1, intermediate_size=64, vocab_size=64,
                      max_position_embeddings=4096, rope_theta=1e6)
    rot = Qwen3RotaryEmbedding(cfg)
    k = torch.randn(1, 2, 11, 128, generator=torch.Generator().manual_seed(0))

    def rope(start):
        p = torch.arange(start, start + k.shape[2])[None]
        cos, sin = rot(k, p)
        return k * cos.unsqueeze(1) + rotate_half(k) * sin.unsqueeze(1)

    out["hf_inv_freq"] = rot.inv_freq.numpy().astype(np.float32)
    out["hf_deltas"] = np.asarray([-7, -1, 0, 1, 13, 64], dtype=np.int64)
    out["hf_k100"] = rope(100).numpy()
    for delta in out["hf_deltas"]:
        out[f"hf_k_{int(delta)}"] = rope(100 + int(delta)).numpy()

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
