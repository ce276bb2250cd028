"""pytest configuration: the ``gpu`` marker and shared fixtures."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter):
    """The largest MoE output errors against the oracle seen in this run."""
    mod = sys.modules.get("tests.test_moe_gpu")
    stats = getattr(mod, "PARITY", None)
    if stats and stats["outputs"]:
        terminalreporter.write_line(
            f"MoE parity: {stats['outputs']} bf16 output rows against the oracle; largest row RMS relative "
            f"error {stats['rms_max']:.3e} (bar {mod.ROW_RMS:g}), largest call RMS {stats['call_rms_max']:.3e} "
            f"(bar {mod.CALL_RMS:g}), largest normwise max error {stats['normwise_max']:.3e} "
            f"(bar 2^-6 = {mod.MAX_NORMWISE:.3e})")
