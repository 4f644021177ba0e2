"""Launch-option registry with the reference's interface (engine/kernels/tune.py:13-48).

The reference times a few launch widths of its small Triton kernels during warmup (``pick``)
and registers each choice as a ``Knob`` that its captured verify step re-judges
(engine/decode.py:556-582, ``knobs``). The B200 kernels have no such options: each derives its
launch shape from the problem shape and the device's SM count (one wave, occupancy-checked
cluster sizes), the same answer in every process, so nothing is timed. ``pick`` therefore
returns the caller's default, and ``knobs`` lists only what a caller registered itself (none
of this package's kernels register any), so the engine's refinement loop has nothing to do.
"""


class Knob:
    """One frozen-at-warmup choice that a captured step can re-judge (engine/kernels/tune.py:31-36)."""

    def __init__(self, name, rows, weight, options, get, select):
        self.name, self.rows, self.weight = name, rows, weight
        self.options, self.get, self.select = options, get, select


_KNOBS = {}


def register(name, rows, weight, options, get, select):
    """Record a choice under ``name`` for the captured step's refinement loop."""
    _KNOBS[name] = Knob(name, rows, weight, options, get, select)


def pick(key, default, options, launch):
    """The launch option for ``key``: always ``default`` (no B200 kernel has alternatives to time)."""
    return default


def knobs(rows):
    """Registered knobs of this row count, largest expected effect first (reference order)."""
    return sorted((knob for knob in _KNOBS.values() if knob.rows == rows), key=lambda knob: -knob.weight)
