"""Shared test setup: puts the package directory (lfm3-kv800_b200/), the repo root (for oracle/) and tests/golden on
sys.path (and the staged reference package after them, when present), and registers the `gpu` marker (tests that need a B200; the CPU suite runs with -m "not gpu")."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "lfm3-kv800_b200"), ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)
# the staged reference package (oracle/stage_reference.py), AFTER this package: the package's pkgutil.extend_path
# then serves the reference modules it does not ship (vllm_attn, torch_decode) over this package's CUDA kv800
REF = os.path.join(ROOT, "oracle", "_ref")
if os.path.isdir(os.path.join(REF, "lfm3_kv800")) and REF not in sys.path:
    sys.path.append(REF)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
