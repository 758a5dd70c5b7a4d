"""CPU: the FMA-pipe exp2 used by the prefill softmax (exp2_fma in
chunked_prefill.cu), restated bit for bit in numpy float32, stays within its
stated 7.5e-5 relative error of exp2 and maps x < -126 (and -inf) to 0."""
import numpy as np

C3, C2, C1, C0 = np.float32(0.05517132), np.float32(0.24261054), np.float32(0.69326097), np.float32(0.99992812)


def exp2_fma(x):
    x = np.asarray(x, dtype=np.float32)
    xc = np.maximum(x, np.float32(-127.0))
    t = (xc + np.float32(12582912.0)).astype(np.float32)
    f = (xc - (t - np.float32(12582912.0))).astype(np.float32)
    p = ((C3 * f + C2) * f + C1) * f + C0
    n = t.view(np.int32) - np.int32(0x4B400000)
    r = (p.astype(np.float32).view(np.int32) + (n << 23)).view(np.float32)
    return np.where(x < -126.0, np.float32(0.0), r)


def test_relative_error_bound():
    x = np.linspace(-125.9, 9.0, 2_000_001, dtype=np.float32)
    got = exp2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 8e-5, rel.max()


def test_masked_and_tiny_inputs_give_zero():
    x = np.array([-np.inf, -1e30, -200.0, -127.0, -126.5], dtype=np.float32)
    assert (exp2_fma(x) == 0).all()
    assert exp2_fma(np.float32(0.0)) == np.float32(exp2_fma(np.float32(0.0)))
    assert abs(float(exp2_fma(np.float32(0.0))) - 1.0) < 1e-4
