"""The addition tree of the router's logits (CPU; no GPU needed).

router_logits_kernel adds the 32 chunk sums of a dot product with a warp xor butterfly (offsets 16, 8, 4, 2, 1;
csrc/exl3b_router.cu), the oracle states the same butterfly (oracle/exl3b_oracle.c ora_router_dot).  The tiled
kernel for many tokens (router_logits_tiled_kernel) instead computes the chunk sums in 5-bit bit-reversed order and
folds each into a 5-level stack like a binary counter.  These tests check, in fp32 numpy arithmetic, that the fold
forms exactly the butterfly's tree: the same result bit for bit, for arbitrary chunk sums.
"""
import numpy as np
import pytest


def butterfly(p: np.ndarray) -> np.float32:
    """Lane 0's value after v[l] = v[l] + v[l ^ o] for o = 16, 8, 4, 2, 1 (every lane ends with the same value)."""
    v = p.astype(np.float32).copy()
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        v = (v + v[lanes ^ o]).astype(np.float32)
    return v[0]


def bitrev5(i: int) -> int:
    return int(format(i, "05b")[::-1], 2)


def counter_fold(p: np.ndarray) -> np.float32:
    """Chunk sums in bit-reversed order; a left subtree waits at its level until its right sibling arrives."""
    stack = [np.float32(0)] * 5
    s = np.float32(0)
    for i in range(32):
        s = np.float32(p[bitrev5(i)])
        for lvl in range(5):
            if (i >> lvl) & 1:
                s = np.float32(stack[lvl] + s)
            else:
                stack[lvl] = s
                break
    return s


@pytest.mark.parametrize("seed", range(8))
def test_fold_equals_butterfly_random(seed):
    rng = np.random.default_rng(seed)
    for _ in range(200):
        scale = 10.0 ** rng.uniform(-6, 6, size=32)   # mixed magnitudes: the tree order decides the rounding
        p = (rng.standard_normal(32) * scale).astype(np.float32)
        assert butterfly(p).view(np.uint32) == counter_fold(p).view(np.uint32)


def test_fold_equals_butterfly_signed_zeros_and_ties():
    cases = [np.zeros(32, np.float32), -np.zeros(32, np.float32), np.full(32, 1e-45, np.float32),
             np.array([(-1.0) ** i * 2.0 ** (i % 24) for i in range(32)], np.float32),
             np.array([1.0 if i % 3 else -1.0 + 2.0 ** -23 for i in range(32)], np.float32)]
    for p in cases:
        assert butterfly(p).view(np.uint32) == counter_fold(p).view(np.uint32)


def test_a_different_order_can_round_differently():
    """Sanity check of the test itself: a plain left-to-right sum of the same chunk sums does not always round
    like the tree (so equality above is not vacuous)."""
    rng = np.random.default_rng(123)
    differs = 0
    for _ in range(200):
        p = (rng.standard_normal(32) * 10.0 ** rng.uniform(-6, 6, size=32)).astype(np.float32)
        seq = np.float32(0)
        for c in range(32):
            seq = np.float32(seq + p[c])
        differs += int(seq.view(np.uint32) != butterfly(p).view(np.uint32))
    assert differs > 0
