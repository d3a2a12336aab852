"""msplat_b200: B200-native engine for msplat's per-iteration training step.

The reference's Python surface (msplat: TrainingConfig, TrainingStats,
Dataset, GaussianTrainer, sync, cleanup, load_dataset) is importable from
here; the names resolve on first use so that building the library needs
none of them.
"""
__version__ = "0.1.0"

_EXPORTS = {
    "TrainingConfig": "trainer", "TrainingStats": "trainer", "GaussianTrainer": "trainer",
    "sync": "trainer", "cleanup": "trainer", "Dataset": "dataset", "load_dataset": "dataset",
}

__all__ = sorted(_EXPORTS)


def __getattr__(name):
    if name in _EXPORTS:
        import importlib
        return getattr(importlib.import_module(f"{__name__}.{_EXPORTS[name]}"), name)
    raise AttributeError(name)
