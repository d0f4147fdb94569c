"""CPU checks of the attention oracles themselves."""
import numpy as np

from oracle import attention as oa


def _qkv(s=200, h=2, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.normal(size=(1, h, s, 128)).astype(np.float32)
    k = (rng.normal(size=(1, h, s, 128)) + 2 * rng.normal(size=(1, h, 1, 128))).astype(np.float32)
    v = rng.normal(size=(1, h, s, 128)).astype(np.float32)
    return q, k, v


def test_sage_oracle_tracks_exact_attention():
    q, k, v = _qkv()
    exact = oa.dense_attention(q, k, v)
    sage = oa.sage_attention(q, k, v)
    assert oa.cosine(sage, exact) > 0.995


def test_sage_oracle_row_subset_matches_full():
    q, k, v = _qkv(s=150)
    full = oa.sage_attention(q, k, v)
    rows = np.array([0, 7, 63, 64, 149])
    part = oa.sage_attention(q, k, v, rows=rows)
    np.testing.assert_array_equal(part, full[:, :, rows])


def test_k_smoothing_is_softmax_invariant():
    # Subtracting a per-channel constant from K shifts each score row by a
    # constant, which softmax ignores: exact attention is unchanged.
    q, k, v = _qkv(s=64)
    shifted = k - k.mean(axis=-2, keepdims=True)
    np.testing.assert_allclose(oa.dense_attention(q, k, v), oa.dense_attention(q, shifted, v),
                               atol=2e-5)


def test_block_quant_roundtrip_error_bound():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(1, 1, 130, 128)).astype(np.float32)
    codes, scales = oa._block_int8(x)
    recon = codes.astype(np.float32) * np.repeat(scales, 64, axis=-1)[..., :130, None]
    assert np.abs(recon - x).max() <= scales.max() / 2 + 1e-7
