"""Stand-in for the reference's ``binary_kernels`` extension module.

The reference builds a torch extension named ``binary_kernels`` whose only job is to
register dispatcher ops (src/nanoquant/kernel/pybind.cpp:83-131,
src/nanoquant/kernel/setup.py:55-74).  Importing this module registers the same op
schemas backed by the sm_100a kernels of this package.
"""
from ._lib import load_torch_ops

load_torch_ops()
