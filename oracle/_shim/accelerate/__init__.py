"""Minimal stand-in for the `accelerate` package, used only so the reference
modules import in the test container (test infrastructure; never shipped).

The reference imports `init_empty_weights` at module top
(prismaquant/export_native_compressed.py:69, prismaquant/layer_streaming.py:25);
neither is on the quantization-cost path.
"""
import contextlib


@contextlib.contextmanager
def init_empty_weights(*args, **kwargs):
    yield
