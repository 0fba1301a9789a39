"""The FMA-pipe exp2 used by the forward kernel's softmax (exp2_poly2 in
csrc/sm100.cuh), evaluated here step for step in float32 numpy: round-to-nearest
split by a 1.5*2^23 add, cubic polynomial for 2^f on [-1/2, 1/2] (fused
multiply-adds in fp32), exponent inserted by an integer add of (bits(t) << 23).
Checked against the exact 2^x over the argument range the kernel uses."""
import numpy as np

C0, C1, C2, C3 = (np.float32(0.9999280571937561), np.float32(0.6932609677314758),
                  np.float32(0.2426111400127411), np.float32(0.0551716573536396))
MAGIC = np.float32(12582912.0)


def fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x):
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + MAGIC).astype(np.float32)
    n = (t - MAGIC).astype(np.float32)
    f = fma32(n, np.float32(-1.0) * np.ones_like(n), x)
    q = fma32(f, np.full_like(f, C3), np.full_like(f, C2))
    q = fma32(q, f, np.full_like(f, C1))
    q = fma32(q, f, np.full_like(f, C0))
    bits = (q.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_over_the_softmax_range():
    x = np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32)
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 8e-5, rel.max()


def test_exact_at_integers_and_tiny_below_range():
    x = np.arange(-120, 9, dtype=np.float32)
    np.testing.assert_allclose(exp2_poly(x), np.exp2(x.astype(np.float64)), rtol=8e-5)
    tiny = exp2_poly(np.array([-200.0, -np.inf, -126.0], np.float32))
    assert np.all(np.isfinite(tiny)) and np.all(tiny <= 2.0 ** -125)
