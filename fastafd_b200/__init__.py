__version__ = "0.1.0"

from .env import apply_reference_aliases as _apply_reference_aliases

_apply_reference_aliases()          # a reference knob that is set (MINISGL_PDL, ...) acts under its new name
