"""ie_tpq -- B200-native tensor-parallel quantized linear layers.

A drop-in for the reference engine's ``ie.parallel`` (sharding and TP layers)
and ``ie.quant`` (formats, quantizer, model driver) on the GPU.  All compute
goes through ``libie_tpq.so`` (hand-written sm_100a CUDA behind a C ABI,
``include/ie_tpq.h``); nothing here computes on the CPU.

Modules mirror the reference:
  ie_tpq.formats        <- ie/quant/formats.py
  ie_tpq.weights        <- ie/quant/weights.py
  ie_tpq.quant_model    <- ie/quant/model.py
  ie_tpq.sharding       <- ie/parallel/sharding.py
  ie_tpq.tensor_parallel<- ie/parallel/tensor_parallel.py (linear path)
and add the device pieces: packed (HBM layouts), linear (the fused kernel
call), comm (the multi-process NVLink communicator).
"""
from ._lib import lib as _native_lib  # noqa: F401

__version__ = "0.1.0"
