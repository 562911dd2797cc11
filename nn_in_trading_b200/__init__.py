"""B200-native re-implementation of the NeuroNet.cl kernel library of EAPrognoz/NN_in_Trading.

The product is the C-ABI shared library libnn_b200.so (include/nn_b200.h) with
hand-written CUDA kernels for sm_100a.  This package holds its sources
(csrc/), the in-tree build (build.py), a ctypes binding mirroring the
reference's COpenCLMy (api.py), and the layer/network sequencing that mirrors
the reference's CNeuron*OCL classes and CNet (layers.py, net.py).
"""
from .api import Context, Kernel, NNError, load_library  # noqa: F401
