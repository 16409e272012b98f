"""The multiply-shift division the attention kernel uses to decode its work units
(csrc/attention.cu, make_fastdiv / fast_div): floor(n / d) == (n * m) >> s for 0 <= n < 2^31,
with l = ceil(log2 d), s = 31 + l, m = ceil(2^s / d) (Granlund and Montgomery 1994, th. 4.2).
Checked here on the integers, for every divisor the kernel's unit decode can meet in practice
and for edge numerators (multiples of d and their neighbours, the top of the range)."""
import numpy as np


def make_fastdiv(d):
    l = 0
    while l < 32 and (1 << l) < d:
        l += 1
    s = 31 + l
    return ((1 << s) + d - 1) // d, s


def test_fastdiv_exact():
    rng = np.random.default_rng(0)
    top = (1 << 31) - 1
    for d in list(range(1, 1025)) + [4095, 4096, 4097, 65535, 65536, 1 << 20, (1 << 31) - 1]:
        m, s = make_fastdiv(d)
        assert m < (1 << 32)
        ks = rng.integers(0, top // d + 1, size=64, dtype=np.int64).tolist() + [0, 1, top // d]
        ns = {top, top - 1, d - 1, d, d + 1}
        for k in ks:
            ns.update(x for x in (k * d - 1, k * d, k * d + 1, k * d + d - 1) if 0 <= x <= top)
        ns.update(rng.integers(0, top + 1, size=256, dtype=np.int64).tolist())
        for n in ns:
            assert (n * m) >> s == n // d, (d, n)
