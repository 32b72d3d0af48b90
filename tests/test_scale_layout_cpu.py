"""CPU checks of the blocked scale-factor layout: the oracle's restatement against a direct
per-byte definition, the round trip, and the C ABI's size and validation logic (no GPU calls)."""
import numpy as np
import pytest

from my_nvfp4_gemm_b200 import capi


def blocked_by_definition(sf):
    rows, cols = sf.shape
    rp, cp = -(-rows // 128) * 128, -(-cols // 4) * 4
    out = np.zeros(rp * cp, dtype=np.uint8)
    for r in range(rows):
        for c in range(cols):
            rb, i, j = r // 128, (r % 128) // 32, r % 32
            cb = c // 4
            out[(rb * (cp // 4) + cb) * 512 + 16 * j + 4 * i + (c % 4)] = sf[r, c]
    return out


@pytest.mark.parametrize("rows,cols", [(1, 1), (128, 4), (130, 5), (256, 16), (97, 33), (300, 64)])
def test_oracle_matches_definition_and_round_trips(oracle, rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    sf = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    b = oracle.scale_to_blocked(sf)
    assert b.size == capi.blocked_scale_bytes(rows, cols)
    assert np.array_equal(b, blocked_by_definition(sf))
    assert np.array_equal(oracle.scale_from_blocked(b, rows, cols), sf)


def test_blocked_sizes():
    assert capi.blocked_scale_bytes(0, 0) == 0
    assert capi.blocked_scale_bytes(1, 1) == 128 * 4
    assert capi.blocked_scale_bytes(8192, 512) == 8192 * 512
    assert capi.blocked_scale_bytes(130, 5) == 256 * 8
    assert capi.blocked_scale_bytes(-1, 4) == -1


def test_validation_before_any_device_work():
    FAKE = 0x10000
    assert capi.scale_to_blocked(FAKE, -1, 4, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.scale_to_blocked(None, 0, 4, None) == capi.NVFP4_OK          # empty: no-op
    assert capi.scale_to_blocked(None, 4, 4, FAKE) == capi.NVFP4_ERR_INVALID_VALUE
    assert capi.scale_to_blocked(FAKE, 4, 4, FAKE + 4) == capi.NVFP4_ERR_MISALIGNED
    assert capi.scale_from_blocked(FAKE + 8, 4, 4, FAKE) == capi.NVFP4_ERR_MISALIGNED
    assert capi.scale_to_blocked(FAKE, 4, 1 << 23, FAKE) == 7               # TOO_LARGE
