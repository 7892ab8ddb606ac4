"""B200-native batched Rocket League tick, a drop-in for the reference's
``carl`` package: re-exports ``Env`` and the upper-case layout constants of the
native module (as the reference's python/carl/__init__.py:11-20 does)."""

from . import carl as _carl

__all__ = [name for name in vars(_carl) if name == "Env" or name.isupper()]
globals().update({name: getattr(_carl, name) for name in __all__})
