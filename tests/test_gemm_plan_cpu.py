"""Dispatch rules of nvfp4_gemm, through the C-ABI's nvfp4_gemm_plan (no device needed when the
SM count is given): which tile and K split each shape runs. The kernels themselves are checked
on the GPU (test_gemm_gpu.py); this pins the choice between them."""
import numpy as np
import pytest

from my_nvfp4_gemm_b200 import capi

B200_SMS = 148


def plan(m, n, k, sms=B200_SMS):
    return capi.gemm_plan(m, n, k, sms)


@pytest.mark.parametrize("m", [129, 256, 1000, 8192])
def test_more_than_128_rows_run_the_cta_pair(m):
    assert plan(m, 8192, 8192) == (256, 256, 1)
    assert plan(m, 3584, 8192) == (256, 256, 1)   # narrow N too: the pair form has no split


@pytest.mark.parametrize("m", [1, 16, 32, 33, 64, 128])
def test_decode_widths_of_a_28672_column_weight(m):
    K = 8192
    assert plan(m, 28672, K) == (128, 256, 1)          # one GPU: 112 tiles of 256 columns
    assert plan(m, 28672 // 2, K) == (128, 128, 1)     # 2 ranks: 112 tiles of 128 columns
    # 4 ranks: 256-column tiles over 4 CTAs at <= 32 rows, 128-column tiles over 2 above
    assert plan(m, 28672 // 4, K) == ((128, 256, 4) if m <= 32 else (128, 128, 2))
    assert plan(m, 28672 // 8, K) == (128, 128, 4)     # 8 ranks: 28 tiles x 4 CTAs


def test_no_split_when_k_is_not_a_multiple_of_the_split():
    # 3 k-blocks: no split divides them; the 3584-column shard falls back to narrower tiles
    assert plan(16, 3584, 768) == (128, 32, 1)
    # 2 k-blocks: a 2-way split only (above 32 rows, 128-column tiles)
    assert plan(100, 7168, 512) == (128, 128, 2)
    assert plan(16, 7168, 512) == (128, 64, 1)


def test_fewer_sms_change_the_choice():
    # a 132-SM part: 28 x 4 = 112 still fits; 56 x 2 = 112 fits; 28672 columns need 112 tiles
    assert plan(16, 3584, 8192, sms=132) == (128, 128, 4)
    assert plan(16, 28672, 8192, sms=132) == (128, 256, 1)
    # very few SMs: nothing is "narrow"
    assert plan(16, 3584, 8192, sms=8) == (128, 256, 1)


def test_plan_invariants_on_random_shapes():
    rng = np.random.default_rng(5)
    for _ in range(3000):
        m = int(rng.integers(1, 300))
        n = int(rng.integers(1, 5000)) * 8
        k = int(rng.integers(1, 80)) * 256
        sms = int(rng.choice([132, 148]))
        tm, tn, ks = plan(m, n, k, sms)
        tiles = lambda bn: -(-n // bn)  # noqa: E731
        assert tm == (256 if m > 128 else 128)
        assert tn in (32, 64, 128, 256) and ks in (1, 2, 4)
        if tm == 256:
            assert (tn, ks) == (256, 1)
            continue
        if tn < 256 or ks > 1:
            assert 2 * tiles(256) <= sms, (m, n, k, sms)   # only shapes that underfill the GPU
        if ks > 1:
            assert tiles(tn) * ks <= sms and (k // 256) % ks == 0, (m, n, k, sms)
            assert ks == 4 or m > 32                        # the 2-way split is for > 32 rows


@pytest.mark.parametrize("m,n,k,status", [(16, 3584, 100, "UNSUPPORTED_SHAPE"),
                                          (16, 3583, 8192, "UNSUPPORTED_SHAPE"),
                                          (-1, 3584, 8192, "INVALID_VALUE"),
                                          (16, 3584, 0, "INVALID_VALUE")])
def test_plan_rejects_what_the_gemm_rejects(m, n, k, status):
    with pytest.raises(RuntimeError, match=status):
        plan(m, n, k)
