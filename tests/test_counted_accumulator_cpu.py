"""Host restatement of the counted fixed-point accumulator words the kernel uses
for its grid-wide sums (layout documented with kAccShift in mkb_config.cuh):
bits 56-63 count contributions, bits 0-55 hold sum(round(x * 2^28) + 2^47).
Checks the invariants the kernel relies on with exact integer arithmetic."""
import random

SHIFT, BIAS, ONE = 28, 1 << 47, 1 << 56
LOW = ONE - 1
LIM = 140737488355000.0  # largest |x * 2^28| the kernel passes on (just below 2^47)


def term(x: float) -> int:
    s = x * (1 << SHIFT)
    s = max(-LIM, min(LIM, s))
    return ONE + int(round(s)) + BIAS


def decode(word_sum: int):
    cnt = word_sum >> 56
    low = word_sum & LOW
    return cnt, (low - cnt * BIAS) / float(1 << SHIFT)


def test_255_extreme_contributions_never_carry_into_the_count():
    for x in (2.0 ** 19 * 0.9999, -(2.0 ** 19) * 0.9999):
        w = sum(term(x) for _ in range(255)) & ((1 << 64) - 1)
        cnt, val = decode(w)
        assert cnt == 255
        assert abs(val - 255 * round(x * 2 ** SHIFT) / 2 ** SHIFT) == 0.0


def test_sum_is_exact_and_order_independent():
    rng = random.Random(0)
    xs = [rng.uniform(-50.0, 50.0) for _ in range(148)]
    w1 = sum(term(x) for x in xs) & ((1 << 64) - 1)
    rng.shuffle(xs)
    w2 = sum(term(x) for x in reversed(xs)) & ((1 << 64) - 1)
    assert w1 == w2
    cnt, val = decode(w1)
    assert cnt == 148
    exact = sum(round(x * 2 ** SHIFT) for x in xs) / 2 ** SHIFT
    assert val == exact
    assert abs(val - sum(xs)) <= 148 * 2.0 ** -(SHIFT + 1)


def test_copies_add_counts_and_values():
    rng = random.Random(1)
    xs = [rng.uniform(-3.0, 3.0) for _ in range(74)]
    copies = [0, 0]
    for i, x in enumerate(xs):
        copies[i % 2] = (copies[i % 2] + term(x)) & ((1 << 64) - 1)
    cnt = sum(c >> 56 for c in copies)
    low = sum(c & LOW for c in copies)
    assert cnt == 74
    assert (low - cnt * BIAS) / 2 ** SHIFT == sum(round(x * 2 ** SHIFT) for x in xs) / 2 ** SHIFT
