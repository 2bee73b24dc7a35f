"""``import swvr`` for code written against pengzhangzhi/swvr.

The reference's public names (``softmax_readout``, ``softmax_readout_mse``,
``SoftmaxReadoutMSE``, ``softmax_readout_reference``, ``__version__``) resolve to this
repository's B200 implementation in ``swvr_b200`` (which adds the fused-norm entry points
``rmsnorm_softmax_readout`` and ``rmsnorm_softmax_readout_mse``); the objects are the same, so
``swvr.softmax_readout is swvr_b200.softmax_readout``.
"""
from swvr_b200 import (SoftmaxReadoutMSE, __version__, rmsnorm_softmax_readout, rmsnorm_softmax_readout_mse,
                       softmax_readout, softmax_readout_mse, softmax_readout_reference)

__all__ = ["softmax_readout", "softmax_readout_mse", "SoftmaxReadoutMSE", "softmax_readout_reference",
           "rmsnorm_softmax_readout", "rmsnorm_softmax_readout_mse"]
