"""A projection's FP32 split-K partials, consumed without a separate merge launch.

Same hand-off as the reference (engine/kernels/merged.py:13-34): a split projection
leaves SPLITS FP32 partial sums per output element; a consumer kernel sums them in split
order, rounds to BF16 and carries on. The CUDA consumers (fb_add_rmsnorm, fb_swiglu,
fb_qk_norm_rope_append) take the partials pointer and split count directly.
"""


class Split:
    """FP32 partials [S, M, N] standing for a BF16 tensor of logical ``shape`` (..., N)."""

    __slots__ = ("partial", "shape")

    def __init__(self, partial, shape):
        self.partial, self.shape = partial, tuple(shape)

    @property
    def splits(self):
        return self.partial.shape[0]

    @property
    def count(self):
        return self.partial.shape[1] * self.partial.shape[2]


def source(x):
    """(tensor to read, SPLITS, elements per split, logical shape) for a tensor or a Split."""
    if isinstance(x, Split):
        return x.partial, x.splits, x.count, x.shape
    return x, 1, 1, tuple(x.shape)
