"""web-engine B200: the quantized-linear / RMSNorm / RoPE hot path of dotstories/web-engine on sm_100a.

The compute lives in libwe_b200.so (CUDA, C ABI: include/we_b200.h); this package is the host-side
mirror of the reference's operator API (src/model/ops.ts over src/gpu/graph.ts) on top of it.
"""
from . import _lib
from .graph import Binding, Buffer, Graph
from .ops import Linear, Mod, Rope, attention, k_split_for, linear, linear_host, no_mod, norm, qk_norm_rotate, rotate
from . import kernels, parallel
from .stream import Streamer
from . import block as blocks
from . import transformer
from . import weights
from . import sequence
from . import comm

__all__ = ["Graph", "Buffer", "Binding", "Linear", "Mod", "Rope", "linear", "linear_host", "norm", "no_mod", "rotate",
           "qk_norm_rotate", "k_split_for", "kernels", "blocks", "transformer", "parallel", "Streamer", "weights", "sequence", "comm", "build"]


def build(verbose: bool = False) -> str:
    """Compiles libwe_b200.so for sm_100a in place (make in csrc/); returns its path."""
    import os
    import subprocess

    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run(["make", "-j8", "-C", os.path.join(here, "csrc")], capture_output=not verbose, text=True)
    if r.returncode != 0:
        raise RuntimeError("building libwe_b200.so failed:\n" + (r.stdout or "") + (r.stderr or ""))
    return _lib.LIB_PATH
