"""Backends: the reference's plug-in surface on the B200 decode path."""

from microgen_b200.backends.b200 import (B200QuantizedBackend, B200TensorParallelBackend,  # noqa: F401
                                         CUDADeviceInfo, PagedKVCache)
from microgen_b200.backends.parallel import (ColumnParallelLinear, RowParallelLinear,  # noqa: F401
                                             apply_tensor_parallelism)
from microgen_b200.backends.quantized import (QuantizedLinear, quantize_linear_layer_per_channel,  # noqa: F401
                                              quantize_model)

__all__ = ["B200QuantizedBackend", "B200TensorParallelBackend", "CUDADeviceInfo", "PagedKVCache",
           "ColumnParallelLinear", "RowParallelLinear", "QuantizedLinear", "quantize_linear_layer_per_channel",
           "quantize_model", "apply_tensor_parallelism"]
