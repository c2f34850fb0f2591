"""gemma4.kt_b200 -- B200 (sm_100a) kernels for gemma4.kt's quantized GEMV and
MoE layer, behind the C ABI of include/g4.h.

Python here is the host-side mirror of the reference's floattensor API
(FloatTensorFactory / FloatTensor.matmul) and MoE block, used by the tests and
the benchmark; the kernels and the runtime live in libg4b200.so.
"""
from ._lib import G4Error, lib, LIB_PATH  # noqa: F401
from .floattensor import (  # noqa: F401
    Context,
    CudaFloatTensor,
    FloatTensorFactory,
    GGMLType,
    UnsupportedOperation,
    QK_K,
    row_shard,
)
from .moe import FfnMoeBlock, MoeLayer, topk  # noqa: F401
from .model import DecoderBatch, DecoderModel, DecoderState, ModelConfig, TensorSource  # noqa: F401
