"""GPU self-test of the exp used for the window-sum terms (exp_term: ex2.approx
with an exactly split argument) against a correctly rounded exp, on a dense
grid of the arguments the sum sees (x = sc - max in [-30, 0]).

The sum decides inv = (float)(1/sum) and so every probability; the test bounds
the term error (max) and, more importantly, its bias weighted by the term
itself, which is what would move the sum systematically."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _eval(x, which):
    import torch
    import quasar_b200 as q
    import ctypes
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    rc = q.lib().quasar_selftest_exp(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                     x.size, which, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_exp_term_error_and_bias():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rs = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-30.0, 0.0, 1 << 22, dtype=np.float32),
                        -rs.exponential(3.0, 1 << 20).astype(np.float32),
                        np.array([0.0, -1e-30, -1e-8, -87.0, -126.0, -200.0, -np.inf], np.float32)])
    fast = _eval(x, 0).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ok = ref > 1e-30
    rel = (fast[ok] - ref[ok]) / ref[ok]
    assert np.abs(rel).max() < 4e-7, np.abs(rel).max()
    bias = float((rel * ref[ok]).sum() / ref[ok].sum())
    assert abs(bias) < 2e-8, bias
    assert fast[-1] == 0.0 and fast[-2] == 0.0  # -200 and -inf flush to 0
    cr = _eval(x, 2).astype(np.float64)
    assert np.abs((cr[ok] - ref[ok]) / ref[ok]).max() < 6e-8  # correctly rounded float
    print("exp_term max rel %.3g weighted bias %.3g" % (np.abs(rel).max(), bias))
