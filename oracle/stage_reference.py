"""Stage the reference's Python sources under oracle/_ref/ -- TEST INFRASTRUCTURE ONLY.

The reference (riceharvest/lfm3-kv800 v0.1.1) is a Python package.  Its "build" for this repository is a copy of its
.py sources, which does not exist on the GPU box unless it travels with the repository snapshot:

    oracle/_ref/lfm3_kv800/*.py     the reference package (its own kv800.py, torch_decode.py, vllm_attn.py, ...;
                                    no prebuilt binaries: lfm3_kv800/_lib/ is not copied)
    oracle/_ref/tests/test_parity.py  the reference's own decode parity test, unmodified

oracle/_ref/ is git-ignored (reference sources never enter this repository's history) and travels to the GPU box
with the working tree.  Users of the staged copy:
  * bench.py --impl reference: the reference's torch_decode.decode on the host cores, imported from oracle/_ref alone
    (its own kv800), in a separate process;
  * tests: the reference's test_parity.py and vllm_attn.py run against this package's CUDA kv800 (this package first
    on sys.path; pkgutil.extend_path in lfm3_kv800/__init__.py adds the staged directory for the modules this package
    does not ship).
Run by __graft_entry__.build() when the reference checkout exists (here, not on the GPU box)."""
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
DEFAULT_SRC = "/root/reference"


def stage(src=None):
    """Copy the reference's package .py files and tests/test_parity.py into oracle/_ref (replacing an older copy).
    Returns the staged root, or None when the reference checkout is absent."""
    src = src or os.environ.get("LFM3KV_REFERENCE_SRC", DEFAULT_SRC)
    pkg = os.path.join(src, "lfm3_kv800")
    if not os.path.isdir(pkg):
        return None
    dst_pkg = os.path.join(OUT, "lfm3_kv800")
    dst_tests = os.path.join(OUT, "tests")
    os.makedirs(dst_pkg, exist_ok=True)
    os.makedirs(dst_tests, exist_ok=True)
    for name in sorted(os.listdir(pkg)):
        if name.endswith(".py"):
            shutil.copyfile(os.path.join(pkg, name), os.path.join(dst_pkg, name))
    shutil.copyfile(os.path.join(src, "tests", "test_parity.py"), os.path.join(dst_tests, "test_parity.py"))
    return OUT


def staged():
    """oracle/_ref if the staged package is present (on the GPU box: if it traveled), else None."""
    return OUT if os.path.exists(os.path.join(OUT, "lfm3_kv800", "torch_decode.py")) else None


if __name__ == "__main__":
    out = stage(sys.argv[1] if len(sys.argv) > 1 else None)
    print(out or "reference checkout not found; nothing staged")
