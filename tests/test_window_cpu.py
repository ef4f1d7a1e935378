"""Host side of the dense sliding window: FA2 window_size -> the C-ABI's (window_q,
window_k), and the oracle's mask against a direct restatement of the definition."""
import numpy as np
import pytest

from tilelang_fa_v100 import _ext
from oracle import attention_ref as R


@pytest.mark.parametrize("window,fields", [((-1, -1), (0, 0)), ((0, -1), (1, 0)), ((255, -1), (256, 0)),
                                           ((-1, 0), (0, 1)), ((100, 50), (101, 51)), (None, (0, 0))])
def test_window_fields(window, fields):
    assert _ext.window_fields(window) == fields


@pytest.mark.parametrize("m,n", [(5, 5), (4, 9), (9, 4)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("window", [(-1, -1), (0, -1), (2, -1), (-1, 0), (1, 3), (3, 1)])
def test_visible_mask_matches_definition(m, n, causal, window):
    left, right = window
    wq, wk = _ext.window_fields(window)
    want = np.zeros((m, n), dtype=bool)
    for i in range(m):
        a = i + n - m
        for j in range(n):
            # the C-ABI's predicate: a - window_q < j and j < a + window_k when set
            ok = (not causal or j <= a) and (wq <= 0 or a - wq < j) and (wk <= 0 or j < a + wk)
            # FA2's: a - left <= j <= a + right
            fa2 = (not causal or j <= a) and (left < 0 or j >= a - left) and (right < 0 or j <= a + right)
            assert ok == fa2
            want[i, j] = ok
    got = R.visible_mask(m, n, causal, window)
    if got is None:
        assert want.all()
    else:
        assert (got == want).all()
