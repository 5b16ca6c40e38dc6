"""Neural models (same names as ``rsl_rl.models``)."""

from .cnn_model import CNNModel
from .mlp_model import MLPModel
from .rnn_model import RNNModel

__all__ = ["CNNModel", "MLPModel", "RNNModel"]
