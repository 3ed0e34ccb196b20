"""k3b200: B200-native routed-expert hot path (placeholder, filled in below)."""
from . import synth  # noqa: F401
