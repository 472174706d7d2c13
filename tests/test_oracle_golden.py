"""Pin the CPU oracle to the reference: every golden vector the reference produced.

The fixtures in ``tests/golden/shift_golden.npz`` were written by running the
reference's own functions (``tests/golden/make_golden.py``).  These tests run
on CPU only and must pass before any GPU parity result means anything.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import shift_oracle as O
from oracle import torch_cpu_path as T

HEADS, D, BS = 8, 128, 16


def _ref_table(golden, delta: int) -> np.ndarray:
    """The reference's own table for ``delta`` in the oracle's ``[2, half]`` form."""
    return np.stack(
        [golden[f"tab_{delta}_emb_cos"][: D // 2], golden[f"tab_{delta}_emb_sin"][: D // 2]]
    ).astype(np.float32)


def _flat_paged(hnd: bool, nblocks: int, dtype=np.uint16):
    shape = (nblocks, HEADS, BS, 2 * D) if hnd else (nblocks, BS, HEADS, 2 * D)
    flat = np.zeros(int(np.prod(shape)), dtype=dtype)
    if hnd:
        blk, head, off = HEADS * BS * 2 * D, BS * 2 * D, 2 * D
    else:
        blk, off, head = BS * HEADS * 2 * D, HEADS * 2 * D, 2 * D
    return O.Paged(flat, 0, D, blk, off, head, BS, HEADS, D)


# ----------------------------------------------------------------- tables
@pytest.mark.parametrize("rot,theta", [(128, 1e6), (64, 1e6), (128, 1e4), (64, 1e4)])
def test_inv_freq_matches_the_connector_expression(golden, rot, theta):
    ref = golden[f"inv_freq_{rot}_{int(theta)}"]
    got = O.inv_freq(rot, theta)
    assert O.ulp_distance(got, ref, O.F32).max() <= 1


def test_angles_are_bit_identical_to_the_reference(golden):
    inv = golden["inv_freq_128_1000000"]
    for d in golden["table_deltas"]:
        assert np.array_equal(O.rope_angles(int(d), inv), golden[f"tab_{int(d)}_ang"]), d


def test_tables_within_one_ulp_of_torch_cos_sin(golden):
    """Correctly rounded cos/sin vs torch's fp32 cos/sin: never more than 1 ulp apart."""
    inv = golden["inv_freq_128_1000000"]
    deltas = golden["table_deltas"]
    mine = O.rope_tables(deltas, inv)
    differing = 0
    for i, d in enumerate(deltas):
        ref = _ref_table(golden, int(d))
        dist = O.ulp_distance(mine[i], ref, O.F32)
        assert dist.max() <= 1, f"delta {d}: {dist.max()} ulp"
        differing += int((dist > 0).sum())
    # record how far the two cos implementations actually drift: a handful of entries
    assert differing <= mine.size // 4


def test_branchless_form_matches_rope_shift_fields(golden):
    for d in golden["table_deltas"]:
        d = int(d)
        cos, sgn, partner = O.branchless_tables(_ref_table(golden, d), D)
        assert np.array_equal(cos, golden[f"tab_{d}_cos"])
        assert np.array_equal(sgn, golden[f"tab_{d}_sgn"])
        assert np.array_equal(partner, golden[f"tab_{d}_partner"])


def test_partial_rotary_tail_is_identity_in_the_tables(golden):
    inv64 = golden["inv_freq_64_1000000"]
    ang = O.rope_angles(37, inv64)
    ref_half = np.stack([golden["partial_cos"][:32], -golden["partial_sgn"][:32]])
    cos, sgn, partner = O.branchless_tables(ref_half.astype(np.float32), 256)
    assert np.array_equal(cos, golden["partial_cos"])
    assert np.array_equal(sgn, golden["partial_sgn"])
    assert np.array_equal(partner, golden["partial_partner"])
    assert np.all(golden["partial_cos"][64:] == 1) and np.all(golden["partial_sgn"][64:] == 0)
    assert O.ulp_distance(O.rope_tables([37], inv64)[0, 0], np.cos(ang.astype(np.float64)).astype(np.float32), O.F32).max() == 0


def test_tables_encode_the_rerotation_identity(golden):
    """Port of the reference's table test (tests/test_shift_kernels.py:32-43) on the oracle."""
    inv = golden["inv_freq_128_1000000"]
    k = np.random.default_rng(0).standard_normal((2, 8, 5, 128)).astype(np.float32)
    for d in (-3000, -4, 0, 4, 186, 10000):
        tab = O.rope_tables([d], inv)[0]
        cos, sgn, partner = O.branchless_tables(tab, D)
        fused = k * cos + k[..., partner] * sgn
        assert np.allclose(fused, O.rotate_keys(k, tab), atol=1e-6)


# ---------------------------------------------------------------- scatter
@pytest.mark.parametrize("delta", [-3000, -4, 0, 4, 186, 10000])
def test_bf16_scatter_is_bit_identical_to_the_reference_given_its_tables(golden, delta):
    src = golden["bf16_src"]
    tab = _ref_table(golden, delta) if delta else None
    k = O.shift_k_bits(src[..., :D], tab, O.BF16)
    assert np.array_equal(k, golden[f"bf16_k_{delta}"])


@pytest.mark.parametrize("delta", [-3000, -4, 0, 4, 186, 10000])
def test_reference_bf16_output_is_its_fp32_rotation_rounded(golden, delta):
    """The golden fp32 rows are the reference's rotation before rounding: its own
    bf16 output is their round-to-nearest-even, bit for bit."""
    assert np.array_equal(O.f32_to_bf16(golden[f"f32r_k_{delta}"]), golden[f"bf16_k_{delta}"])


@pytest.mark.parametrize("delta", [-3000, -4, 0, 4, 186, 10000])
def test_bf16_scatter_with_own_tables_is_within_one_ulp_of_the_reference(golden, delta):
    """The north star's bar, element by element and with no allowance: with the
    oracle's own (correctly rounded) tables, every K element is within one bf16
    ulp of the reference's fp32 rotation, computed with the reference's tables."""
    src = golden["bf16_src"]
    inv = golden["inv_freq_128_1000000"]
    tab = O.rope_tables([delta], inv)[0] if delta else None
    k = O.shift_k_bits(src[..., :D], tab, O.BF16)
    ok = O.within_one_step(k, golden[f"f32r_k_{delta}"], O.BF16)
    assert ok.all(), f"{int((~ok).sum())} of {ok.size} K elements beyond one ulp"
    # and against the reference's rounded output: at most one ulp apart
    assert O.ulp_distance(k, golden[f"bf16_k_{delta}"], O.BF16).max() <= 1


def test_one_step_bar_rejects_a_two_ulp_error(golden):
    """The bar is not vacuous: both bf16 neighbours of r pass it (r lies between
    them), a value two codes above the nearest one fails it."""
    r = golden["f32r_k_186"]
    k = O.f32_to_bf16(r)
    pos = (O.bf16_to_f32(k) > 0) & (r > 0)
    r, k = r[pos], k[pos]
    assert O.within_one_step(k, r, O.BF16).all()
    other = np.where(O.bf16_to_f32(k) <= r, k.astype(np.int32) + 1, k.astype(np.int32) - 1)
    assert O.within_one_step(other.astype(np.uint16), r, O.BF16).all()
    off2 = (k.astype(np.int32) + 2).astype(np.uint16)
    assert not O.within_one_step(off2, r, O.BF16).any()


def test_e4m3_one_step_bar():
    r = np.array([1.0, 1.0624, 0.0009, 447.0, 500.0, -3.3], dtype=np.float32)
    q = O.f32_to_e4m3(r)
    assert O.within_one_step(q, r, O.E4M3).all()
    nxt = O.f32_to_e4m3(O.e4m3_to_f32(q) * np.float32(1.3))  # about two steps up
    assert not O.within_one_step(nxt, r, O.E4M3)[[0, 5]].any()


def test_fast_e4m3_rounding_matches_its_definition():
    """The oracle's integer-arithmetic e4m3 rounding equals nearest-code search
    (ties to even, saturation at 448) on every 97th fp32 pattern up to 448,
    every code, every midpoint and its neighbours."""
    u = np.arange(0, 0x43E00001, 97 * 11, dtype=np.uint32)
    mids = (O._E4M3[:-1] + O._E4M3[1:]) / 2
    x = np.concatenate([u.view(np.float32), O._E4M3.astype(np.float32),
                        mids.astype(np.float32), np.nextafter(mids.astype(np.float32), 0),
                        np.nextafter(mids.astype(np.float32), np.float32(1e3)),
                        np.float32([500.0, 1e30, 0.0])])
    x = np.concatenate([x, -x])
    assert np.array_equal(O.f32_to_e4m3(x), O._f32_to_e4m3_by_search(x))


@pytest.mark.parametrize("hnd", [True, False])
def test_placement_through_slots_both_layouts(golden, hnd):
    src = golden["bf16_src"]
    slots = golden["bf16_slots"]
    paged = _flat_paged(hnd, 64)
    tab = _ref_table(golden, 186)
    O.scatter_shifted(src, paged, slots, tab, O.BF16)
    k, v = paged.read(slots)
    assert np.array_equal(k, golden["bf16_k_186"])
    assert np.array_equal(v, src[..., D:])
    written = np.zeros(paged.flat.size, dtype=bool)
    written[paged._index(paged.k_base, slots)] = True
    written[paged._index(paged.v_base, slots)] = True
    assert not paged.flat[~written].any()


@pytest.mark.parametrize("delta", [0, 1, -1, 17, -17, 566, -566, -1133, 6759])
@pytest.mark.parametrize("hnd", [True, False])
def test_fp32_qwen3_geometry_digest(golden, delta, hnd):
    """fp32 rows land bit-identical to the reference's scatter (test_shift_kernels.py:93-134)."""
    src = O.bf16_to_f32(golden["bf16_src"])
    slots = golden["f32_slots"]
    paged = _flat_paged(hnd, 12, dtype=np.float32)
    tab = _ref_table(golden, delta) if delta else None
    O.scatter_shifted(src, paged, slots, tab, O.F32)
    k, v = paged.read(slots)
    rows = np.concatenate([k, v], axis=-1).astype(np.float32)
    digest = hashlib.sha256(np.ascontiguousarray(rows).tobytes()).digest()
    tag = f"{delta}_{'hnd' if hnd else 'nhd'}"
    assert digest == golden[f"f32_digest_{tag}"].tobytes()


def test_negative_control_a_wrong_angle_is_caught(golden):
    """Delta 100 vs 101 must not agree (tests/test_shift_kernels.py:137-155)."""
    inv = golden["inv_freq_128_1000000"]
    k = O.bf16_to_f32(golden["bf16_src"][..., :D])
    a = O.rotate_keys(k, O.rope_tables([100], inv)[0])
    b = O.rotate_keys(k, O.rope_tables([101], inv)[0])
    assert not np.allclose(a, b, atol=1e-4)


def test_rotation_composes_additively(golden):
    """rotate(rotate(k, d1), d2) == rotate(k, d1 + d2) up to angle rounding (remap's premise).

    Each angle ``fp32(d * f)`` carries a rounding error of at most half an
    ulp of ``|d| * f <= |d|``, so the two paths differ by at most the sum of
    those errors (times |k|) plus fp32 arithmetic noise.
    """
    inv = golden["inv_freq_128_1000000"]
    k = O.bf16_to_f32(golden["bf16_src"][..., :D])
    kmax = float(np.abs(k).max())
    for d1, d2 in ((37, 180), (-566, 600), (10000, -9999)):
        t1, t2, t12 = (O.rope_tables([d], inv)[0] for d in (d1, d2, d1 + d2))
        two = O.rotate_keys(O.rotate_keys(k, t1), t2)
        one = O.rotate_keys(k, t12)
        angle_err = (abs(d1) + abs(d2) + abs(d1 + d2)) * 2.0**-24
        assert np.abs(two - one).max() <= 2 * (angle_err + 8 * 2.0**-24) * kmax


def test_hf_qwen3_rotary_identity(golden):
    """rerotate(K@p, delta) == K@(p+delta) through transformers' own rotary (test_kvshift.py:48-55)."""
    inv = golden["hf_inv_freq"]
    base = golden["hf_k100"]
    for d in golden["hf_deltas"]:
        d = int(d)
        got = O.rotate_keys(base, O.rope_tables([d], inv)[0])
        assert np.allclose(got, golden[f"hf_k_{d}"], atol=1e-5, rtol=1e-4), d


# ----------------------------------------------------------------- slots
def test_slots_known_answer(golden):
    assert O.slots([7, 3], 2, 6, 4).tolist() == [30, 31, 12, 13]
    assert np.array_equal(O.slots([7, 3], 2, 6, 4), golden["slots_known"])


def test_slots_block_table(golden):
    assert np.array_equal(O.slots(golden["slots_bt"], 1061, 4133, 16), golden["slots_bt_out"])


# --------------------------------------------------------------- rounding
def test_bf16_rounding_matches_torch(golden):
    assert np.array_equal(O.f32_to_bf16(golden["round_in"]), golden["round_bf16"])


def test_f16_rounding_matches_torch(golden):
    assert np.array_equal(O.f32_to_f16(golden["round_in"]), golden["round_f16"])


def test_e4m3_rounding_matches_torch(golden):
    assert np.array_equal(O.f32_to_e4m3(golden["round_e4m3_in"]), golden["round_e4m3"])


def test_e4m3_decode_roundtrip():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    assert np.array_equal(O.f32_to_e4m3(O.e4m3_to_f32(codes)), np.where(codes == 0x80, 0x80, codes))


# --------------------------------------------------- the timed CPU baseline
@pytest.mark.parametrize("hnd", [True, False])
def test_torch_cpu_path_equals_the_numpy_oracle(golden, hnd):
    src_bits = golden["bf16_src"]
    slots = golden["bf16_slots"]
    tab = _ref_table(golden, 186)
    src = torch.from_numpy(src_bits.view(np.int16).copy()).view(torch.bfloat16)
    shape = (64, HEADS, BS, 2 * D) if hnd else (64, BS, HEADS, 2 * D)
    kv = torch.zeros(shape, dtype=torch.bfloat16)
    T.scatter_layer(src, kv, torch.from_numpy(slots), BS, hnd, T.emb_tables(torch.from_numpy(tab)))
    paged = _flat_paged(hnd, 64)
    O.scatter_shifted(src_bits, paged, slots, tab, O.BF16)
    assert np.array_equal(kv.view(torch.int16).numpy().view(np.uint16).reshape(-1), paged.flat)


def test_save_then_unshifted_load_is_identity():
    rng = np.random.default_rng(3)
    heads, d, bs, nblk = 2, 16, 4, 10
    flat = rng.integers(0, 2**16, nblk * bs * heads * 2 * d, dtype=np.uint16)
    paged = O.Paged(flat.copy(), 0, d, bs * heads * 2 * d, heads * 2 * d, 2 * d, bs, heads, d)
    store = [[np.zeros((40, heads, 2 * d), dtype=np.uint16)]]
    run = {"session": 0, "store_start": 5, "len": 13, "block_table": [3, 1, 7, 9], "paged_start": 2}
    O.save(store, [run], [paged])
    paged.flat[:] = 0
    O.load(store, [dict(run, table=-1)], [paged], [], O.BF16)
    idx = O.run_slots(run, 13, bs)
    k, v = paged.read(idx)
    k0, v0 = O.Paged(flat, 0, d, bs * heads * 2 * d, heads * 2 * d, 2 * d, bs, heads, d).read(idx)
    assert np.array_equal(k, k0) and np.array_equal(v, v0)


def test_torch_cpu_e4m3_path_equals_the_numpy_oracle(golden):
    """The e4m3 CPU baseline (dequantise, rotate, divide, saturate) is the oracle, bit for bit."""
    rng = np.random.default_rng(8)
    n = 40
    vals = (rng.standard_normal((n, HEADS, 2 * D)) * 60).clip(-448, 448).astype(np.float32)
    codes = O.f32_to_e4m3(vals)
    slots = golden["bf16_slots"]
    tab = O.rope_tables([-566], golden["inv_freq_128_1000000"])[0]
    k_scale = 0.0371
    src = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn)
    kv = torch.zeros((64, BS, HEADS, 2 * D), dtype=torch.float8_e4m3fn)
    T.scatter_layer_e4m3(src, kv, torch.from_numpy(slots), BS, False,
                         T.emb_tables(torch.from_numpy(tab)), k_scale)
    paged = _flat_paged(False, 64, dtype=np.uint8)
    O.scatter_shifted(codes, paged, slots, tab, O.E4M3, k_scale)
    assert np.array_equal(kv.view(torch.uint8).numpy().reshape(-1), paged.flat)
