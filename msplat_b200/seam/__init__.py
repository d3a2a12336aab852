"""The reference's backend seam (core/metal/bindings.h) on the CUDA engine;
build_seam.py compiles the reference's Model, Trainer and C API over it."""
