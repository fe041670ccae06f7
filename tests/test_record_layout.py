"""Stage-record layout of the decode GEMV, checked on the CPU.

The numpy model (record_layout.py) of the record build and of the kernel's bf16 pair arithmetic
must give back every weight's s*m*2^e exactly — for every sign/mantissa combination, every
exponent the compressor emits (-27 .. -3) and beyond, and partial 128-row groups — must keep
every outlier (row, column, fp16 value) of the reference's COO list, and must agree with the
oracle's dequantisation (times 15) on a reference-generated fixture.
"""
import numpy as np
import pytest

from oracle import oabf
from golden_io import load
import record_layout as RL


def _exact(exps, signs, payload, npad, kpad):
    sgn, mant, e = oabf.unpack_fields(exps, signs, payload)
    v = np.where(sgn == 1, -mant, mant).astype(np.float64) * np.exp2(e.astype(np.float64))[:, None]
    return v.reshape(npad, kpad)


def _random_packed(npad, kpad, seed, e_lo=-27, e_hi=-3):
    rng = np.random.default_rng(seed)
    nb = npad * kpad // 16
    exps = rng.integers(e_lo, e_hi + 1, size=nb).astype(np.int8)
    signs = rng.integers(-32768, 32768, size=nb).astype(np.int16)
    payload = rng.integers(-2**31, 2**31, size=(nb, 2), dtype=np.int64).astype(np.int32)
    return exps, signs, payload


@pytest.mark.parametrize("npad,kpad,seed", [(192, 512, 0), (128, 256, 1), (64, 768, 2)])
def test_records_decode_exactly(npad, kpad, seed):
    exps, signs, payload = _random_packed(npad, kpad, seed)
    rec = RL.build_records(exps, signs, payload, npad, kpad)
    units = RL.n_units(npad, kpad)
    assert rec.size == RL.table_bytes(units) + units * RL.ENT_OFF
    got = RL.decode_records(rec, npad, kpad).astype(np.float64)
    np.testing.assert_array_equal(got, _exact(exps, signs, payload, npad, kpad))


def test_records_every_field_value_and_exponent_range():
    """Every (sign, mantissa) in every element position, exponents from -128 to 120."""
    npad, kpad = 128, 256
    nb = npad * kpad // 16
    el = np.arange(16)
    m = (np.arange(nb)[:, None] + el[None, :]) % 16
    s = ((np.arange(nb)[:, None] // 16 + el[None, :]) % 2).astype(np.int64)
    payload = np.zeros((nb, 2), dtype=np.int64)
    for i in range(8):
        payload[:, 0] |= m[:, i] << (4 * i)
        payload[:, 1] |= m[:, 8 + i] << (4 * i)
    payload = payload.astype(np.uint32).view(np.int32)
    signs = (s << el[None, :]).sum(axis=1).astype(np.uint16).view(np.int16)
    exps = (np.arange(nb) % 249 - 128).astype(np.int8)           # -128 .. 120
    rec = RL.build_records(exps, signs, payload, npad, kpad)
    got = RL.decode_records(rec, npad, kpad).astype(np.float64)
    np.testing.assert_array_equal(got, _exact(exps, signs, payload, npad, kpad))


def test_records_match_oracle_on_reference_fixture():
    g = load("decode_t3_bf16")                                    # 192 x 256, reference-generated
    kpad, npad = g["padded_shape"]
    n, k = g["orig_shape"]
    tiles = RL.outlier_tiles(g["block_idx"], g["offset"], g["value_bits"], npad, kpad, n, k)
    rec = RL.build_records(g["exponents"], g["signs"], g["payload"], npad, kpad, tiles)
    got = RL.decode_records(rec, npad, kpad)
    deq = oabf.dequantize_dense(g["exponents"], g["signs"], g["payload"], g["padded_shape"],
                                g["orig_shape"], crop=False).astype(np.float64)
    # the kernel holds s*m*2^e and applies the format's 1/15 once to the accumulator
    np.testing.assert_allclose(got.astype(np.float64) / 15.0, deq, rtol=2e-7, atol=0)
    # every outlier of the reference's COO list is in the records, at its row and column
    r, c, v = RL.decode_outliers(rec, npad, kpad)
    gi = g["block_idx"].astype(np.int64) * 16 + g["offset"].astype(np.int64)
    np.testing.assert_array_equal(r, gi // kpad)
    np.testing.assert_array_equal(c, gi % kpad)
    np.testing.assert_array_equal(v, g["value_bits"].astype(np.int64) & 0xFFFF)
    assert g["count"] > 0
