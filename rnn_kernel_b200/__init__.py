"""B200-native FP32 GRU training path with an ``nn.GRU``-compatible surface.

Importing the package needs neither a GPU nor the CUDA library; the library
(``librnn_kernel_b200.so``, built in-tree) is loaded on first use.
"""
from .gru import (
    GRU,
    GRUFunction,
    MAX_HIDDEN_SIZE,
    from_torch_gru,
    gru_forward_inference,
    is_b200_available,
    is_supported_gru,
)
from .loss import MSELossFunction, mse_loss
from .train import DataParallelTrainer, GraphedTrainStep, HostBatchPrefetcher, flatten_parameters_

B200GRU = GRU

__all__ = [
    "GRU",
    "B200GRU",
    "GRUFunction",
    "MAX_HIDDEN_SIZE",
    "DataParallelTrainer",
    "GraphedTrainStep",
    "HostBatchPrefetcher",
    "flatten_parameters_",
    "from_torch_gru",
    "gru_forward_inference",
    "is_b200_available",
    "is_supported_gru",
    "mse_loss",
    "MSELossFunction",
]
