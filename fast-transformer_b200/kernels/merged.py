"""A projection's FP32 split-K partials, consumed without a separate merge launch.

Same hand-off as the reference (engine/kernels/merged.py:13-34): a split projection
leaves SPLITS FP32 partial sums per output element; a consumer kernel sums them in split
order, rounds to BF16 and carries on. The CUDA consumers (fb_add_rmsnorm, fb_swiglu,
fb_swiglu_blocked, fb_qk_norm_rope_append, fb_reduce_push) take the partials pointer and split
count directly.

The engine tells a Split from a tensor with ``isinstance`` and reads ``.partial`` and ``.shape``,
and ``source`` answers with the same 4-tuple as the reference's, so those names stay.
"""


class Split:
    """Stands in for a BF16 tensor of logical shape ``shape`` (..., N) that has not been
    rounded yet: ``partial`` holds its S FP32 K-split sums as [S, M, N], M * N = the logical
    element count."""

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
    """What a consumer kernel reads for ``x``: (buffer, split count, elements per split slab,
    logical shape). A plain tensor is one slab of itself."""
    if isinstance(x, Split):
        return x.partial, x.splits, x.count, x.shape
    return x, 1, 1, tuple(x.shape)
