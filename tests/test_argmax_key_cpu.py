"""Host restatement of the 64-bit argmax key the kernel reduces with red.max
across CTAs (argmax_key in mkb_decode.cu): order-preserving bits of the FP32
value (every NaN as one value above +inf, -0 as +0) over the complement of the
row index. The largest key must be torch.argmax's choice: the maximum value,
the first index among equal values, and the first NaN if there is one."""
import numpy as np
import torch


def key(v: float, i: int) -> int:
    f = np.float32(v)
    if np.isnan(f):
        u = 0x7FC00000
    elif f == 0.0:
        u = 0
    else:
        u = int(np.array([f], dtype=np.float32).view(np.uint32)[0])
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - i)


def index(k: int) -> int:
    return 0xFFFFFFFF - (k & 0xFFFFFFFF)


def key_argmax(x: np.ndarray) -> int:
    # the kernel's reduction: per-CTA maxima of the keys, then the max over CTAs
    return index(max(max(key(float(v), i) for i, v in enumerate(x) if i % 148 == c) for c in range(min(148, len(x)))))


def check(x: np.ndarray):
    assert key_argmax(x) == int(torch.argmax(torch.from_numpy(x)))


def test_random_values_match_torch():
    rng = np.random.default_rng(0)
    for n in (1, 7, 148, 1000):
        check(rng.standard_normal(n).astype(np.float32))


def test_ties_take_the_first_index():
    x = np.zeros(300, dtype=np.float32)
    x[17] = x[250] = x[299] = 3.5
    check(x)
    check(np.full(200, -2.0, dtype=np.float32))


def test_signed_zeros_tie():
    x = np.array([-0.0, 0.0, -1.0], dtype=np.float32)
    check(x)
    check(np.array([-1.0, 0.0, -0.0], dtype=np.float32))


def test_nan_is_the_maximum_and_first_nan_wins():
    x = np.array([1.0, np.inf, np.nan, 5.0, np.nan], dtype=np.float32)
    check(x)
    neg_nan = np.array([0x7FC00001 | 0x80000000], dtype=np.uint32).view(np.float32)[0]
    y = np.array([np.inf, neg_nan, 2.0], dtype=np.float32)
    check(y)


def test_infinities_and_empty_candidates():
    x = np.array([-np.inf, -np.inf, -3e38], dtype=np.float32)
    check(x)
    # a CTA without rows offers (-inf, INT_MAX); every real candidate beats it,
    # and the reset value 0 is below every key
    assert key(float("-inf"), 2**31 - 1) < key(float("-inf"), 5)
    assert 0 < key(float("-inf"), 2**31 - 1)
