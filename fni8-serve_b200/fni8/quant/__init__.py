"""Weight quantisation helpers (`fni8.quant.core`, `fni8.quant.lowbit`)."""
from . import core, lowbit  # noqa: F401
