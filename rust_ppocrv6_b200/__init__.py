"""B200-native (sm_100a) quantised recognition head of rust-ppocrv6.

The W8A32 projection of SVTR features onto the CTC vocabulary (MatMul.12 + Add.204),
softmax (Softmax.2) and the per-timestep greedy argmax, as hand-written tcgen05/TMEM CUDA
kernels behind the C ABI in include/rechead.h, plus the CTC collapse (host or GPU) and the
batched recognition preprocessing that produces the network's input (RecPreprocess).
Everything here runs through librechead.so; there is no CPU fallback.
"""
from ._lib import (RH_ERR_CUDA, RH_ERR_DEVICE_FAULT, RH_ERR_INVALID_ARG, RH_ERR_NO_DEVICE, RH_ERR_TIMEOUT,
                   RH_ERR_UNSUPPORTED, RH_OK, RecHeadError, header_symbols, load)
from .ctc import CtcDecoder
from .preprocess import RecPreprocess, batch_shape, rec_preprocess_device, resized_width
from .head import (Context, Fp32Weight, QuantizedWeight, ctc_collapse_device, default_context, head_decode,
                   head_decode_ctc, head_decode_device, head_decode_kt, head_decode_kt_ctc, matmul_quantized_b,
                   matmul_quantized_b_device,
                   matmul_transposed_b)

__all__ = [
    "Context", "QuantizedWeight", "Fp32Weight", "CtcDecoder", "RecHeadError",
    "matmul_quantized_b", "matmul_transposed_b", "head_decode", "head_decode_kt", "head_decode_kt_ctc",
    "head_decode_ctc",
    "head_decode_device", "matmul_quantized_b_device", "ctc_collapse_device",
    "default_context", "load", "header_symbols",
    "RecPreprocess", "resized_width", "batch_shape", "rec_preprocess_device",
    "RH_OK", "RH_ERR_INVALID_ARG", "RH_ERR_CUDA", "RH_ERR_TIMEOUT", "RH_ERR_UNSUPPORTED", "RH_ERR_NO_DEVICE",
    "RH_ERR_DEVICE_FAULT",
]
