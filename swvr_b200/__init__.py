"""swvr_b200: ``softmax(h @ W.T + b) @ E`` (and an MSE loss on it) on B200 without materialising ``[N, V]``.

A drop-in for pengzhangzhi/swvr (``import swvr_b200 as swvr``) whose compute runs in
hand-written sm_100a kernels (libswvr_b200.so, C ABI in include/swvr_b200.h).
"""
from .api import SoftmaxReadoutMSE, softmax_readout, softmax_readout_mse
from .norm import rmsnorm_softmax_readout, rmsnorm_softmax_readout_mse
from .reference import softmax_readout_reference

__all__ = ["softmax_readout", "softmax_readout_mse", "SoftmaxReadoutMSE", "softmax_readout_reference",
           "rmsnorm_softmax_readout", "rmsnorm_softmax_readout_mse"]
__version__ = "0.1.0"
