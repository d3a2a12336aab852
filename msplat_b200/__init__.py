"""msplat_b200: B200-native engine for msplat's per-iteration training step."""
__version__ = "0.1.0"
