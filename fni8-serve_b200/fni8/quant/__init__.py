"""Weight quantisation helpers (`fni8.quant.core`)."""
from . import core  # noqa: F401
