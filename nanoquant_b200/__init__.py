"""B200-native (sm_100a) kernels for NanoQuant's quantized-linear inference path.

Importing the package registers the dispatcher ops (``torch.ops.binary_kernels.*`` with
the reference schemas and ``torch.ops.nq_b200.*``) and makes ``import binary_kernels``
resolve to them, which is what the reference's ``get_kernel_function`` and
``_prepare_kernel`` import (src/nanoquant/kernel/utils.py:33-48, modules/linear.py:235).
"""
import sys

from . import _lib
from ._lib import NQError, cuda_lib, load_torch_ops

load_torch_ops()

from . import binary_kernels  # noqa: E402
from .kernel_utils import (binary_packer, binary_unpacker, get_kernel_function, pack_binary_gemv,  # noqa: E402
                           repack_binary, unpack_binary_gemv)
from .linear import NanoQuantLinear  # noqa: E402

sys.modules.setdefault("binary_kernels", binary_kernels)

__all__ = ["NanoQuantLinear", "NQError", "binary_packer", "binary_unpacker", "cuda_lib", "get_kernel_function",
           "load_torch_ops", "pack_binary_gemv", "repack_binary", "unpack_binary_gemv"]
