"""GPU self-test of the exp used for the terms of the window sum against a
correctly rounded exp, on a dense grid of the arguments the sum sees
(x = sc - max in [-30, 0] and beyond).

The window sum decides inv = (float)(1/sum) and so every probability, so the
test bounds the term error (max) and, more importantly, its bias weighted by
the term itself - a systematic error would move the sum of ~1e5 terms and so
every probability. The default term (which 4: ex2.approx of x*log2e, one
multiply and one MUFU op) must stay far inside the 1e-5 relative tolerance on
p and the 1e-6 band on cumulative sums; the FMA-pipe polynomial (which 3) is
the more accurate, slower alternative."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _eval(x, which):
    import torch
    import quasar_b200 as q
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    rc = q.lib().quasar_selftest_exp(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                     x.size, which, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def grid():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rs = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-30.0, 0.0, 1 << 22, dtype=np.float32),
                        -rs.exponential(3.0, 1 << 20).astype(np.float32),
                        np.array([0.0, -1e-30, -1e-8, -80.0, -86.0, -200.0, -np.inf], np.float32)])
    return x, np.exp(x.astype(np.float64))


def _stats(fast, ref):
    ok = ref > 1e-30
    rel = (fast[ok] - ref[ok]) / ref[ok]
    return np.abs(rel).max(), float((rel * ref[ok]).sum() / ref[ok].sum())


def test_sum_exp_error_and_bias(grid):
    x, ref = grid
    fast = _eval(x, 4).astype(np.float64)
    mx, bias = _stats(fast, ref)
    print("exp_fast max rel %.3g weighted bias %.3g" % (mx, bias))
    # product rounding: |x log2e| * 2^-24 * ln2 relative, largest at x = -30
    assert mx < 5e-6, mx
    assert abs(bias) < 1e-7, bias
    assert fast[x.size - 7] == 1.0      # exp(0) is exact
    assert fast[-1] == 0.0 and fast[-2] < 1e-37


def test_poly_exp_error_and_bias(grid):
    x, ref = grid
    fast = _eval(x, 3).astype(np.float64)
    mx, bias = _stats(fast, ref)
    print("exp_poly max rel %.3g weighted bias %.3g" % (mx, bias))
    assert mx < 2.5e-7, mx
    assert abs(bias) < 5e-9, bias
    assert fast[x.size - 7] == 1.0      # exp(0) is exact
    assert fast[-1] < 1e-37 and fast[-2] < 1e-37


def test_other_exp_variants(grid):
    x, ref = grid
    mx0, b0 = _stats(_eval(x, 0).astype(np.float64), ref)
    print("ex2.approx split: max rel %.3g weighted bias %.3g" % (mx0, b0))
    assert mx0 < 4e-7
    mx1, b1 = _stats(_eval(x, 1).astype(np.float64), ref)
    print("expf: max rel %.3g weighted bias %.3g" % (mx1, b1))
    assert mx1 < 2.5e-7
    mx2, _ = _stats(_eval(x, 2).astype(np.float64), ref)
    assert mx2 < 6e-8  # correctly rounded float
