"""The power-of-two scaling a bf16 query takes before the f16 products of fp8-cache decode
(`fa_decode.cu`, the `q_up` / `q_down` block), restated in numpy: the exponent of the
group's largest |q| picks qk = 141 - biased_exponent, clamped to [-100, 100].  Checked
here: the scaled maximum lies in [2^14, 2^15) unless the clamp binds, every element down
to 2^-28 of the maximum converts to f16 exactly, and scaling back by 2^-qk restores it."""
import numpy as np
import pytest


def _bf16(x):
    """Round float32 to bfloat16 (nearest even), returned as float32."""
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def _raw_qk(group):
    amax = np.float32(np.max(np.abs(group)))
    return 141 - int((amax.view(np.uint32) >> 23) & 0xFF)


def _qk(group):
    return max(-100, min(100, _raw_qk(group)))


@pytest.mark.parametrize("magnitude", [1e-30, 1e-6, 1e-2, 1.0, 37.0, 3e5, 1e20])
def test_scaled_group_is_exact_in_f16(magnitude):
    rng = np.random.default_rng(int(np.log2(magnitude) + 200))
    q = _bf16(rng.standard_normal(4 * 256).astype(np.float32) * np.float32(magnitude))
    qk = _qk(q)
    up = np.float32(2.0 ** qk)
    scaled = q * up
    amax = np.max(np.abs(scaled))
    h = scaled.astype(np.float16)
    if _raw_qk(q) <= 100:
        assert 2.0 ** 14 <= amax < 2.0 ** 15
        big = np.abs(q) >= np.max(np.abs(q)) * 2.0 ** -28
    else:  # the clamp binds (largest |q| below 2^-86): exact down to f16's normal range
        assert amax < 2.0 ** 14
        big = np.abs(scaled) >= 2.0 ** -14
    assert np.array_equal(h[big].astype(np.float32), scaled[big])
    assert np.array_equal(h[big].astype(np.float32) * np.float32(2.0 ** -qk), q[big])
    # products with e4m3 values (|k| <= 448) summed over 512 dims stay far inside f32
    assert amax * 448 * 512 < 2.0 ** 40


def test_zero_group_and_clamp():
    assert _qk(np.zeros(8, np.float32)) == 100      # all zeros: any scale, clamped
    assert _qk(np.array([np.inf], np.float32)) == -100
    assert _qk(np.array([1.0], np.float32)) == 14
    assert _qk(np.array([2.0 ** 14], np.float32)) == 0
