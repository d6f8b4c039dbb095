"""800h KV cache for LiquidAI LFM3 on B200 (sm_100a): the reference package's operator surface (lfm3_kv800) over one
hand-written CUDA backend reached through a plain C ABI (include/kv800_b200.h).

Modules: kv800 (cache layout, quantizer / flush, decode dispatch, PagedStore), ops (torch.ops.kv800, the reference's
op schema), train (fake quantization and the training hook patch_for_training), vllm_step (the vLLM decode step on
the device), dp (sequence sharding), _lib (ctypes binding of the CUDA library).  Kept free of torch imports so that importing the package is cheap (the reference's convention,
lfm3_kv800/__init__.py:1-6)."""
import logging
import pkgutil

# Drop-in with the reference installed beside this package: other `lfm3_kv800` directories on sys.path (after this
# one) join the package, so the modules this build does not ship -- the reference's vllm_attn, vllm_model, plugin,
# torch_decode -- import from there, while kv800, train and ops resolve to this directory first.  Their
# `from . import kv800` then binds this package's CUDA kv800.
__path__ = pkgutil.extend_path(__path__, __name__)

__version__ = "0.1.1+b200"


def get_logger() -> logging.Logger:
    """Package logger that prints INFO lines in every process (lfm3_kv800/__init__.py:12-21 of the reference)."""
    lg = logging.getLogger("lfm3_kv800")
    if not lg.handlers:
        h = logging.StreamHandler()
        h.setFormatter(logging.Formatter("%(levelname)s %(asctime)s [lfm3_kv800] %(message)s", "%m-%d %H:%M:%S"))
        lg.addHandler(h)
        lg.setLevel(logging.INFO)
        lg.propagate = False
    return lg
