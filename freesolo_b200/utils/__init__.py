"""Host-side mirror of the reference's ``src.utils`` names used around the attention hot path."""
from . import trunk_triton  # noqa: F401
