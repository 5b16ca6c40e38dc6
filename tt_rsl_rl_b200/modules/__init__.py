"""Building blocks for neural models (same names as ``rsl_rl.modules``)."""

from .cnn import CNN
from .distribution import BetaDistribution, Distribution, GaussianDistribution, HeteroscedasticGaussianDistribution
from .mlp import MLP
from .normalization import EmpiricalDiscountedVariationNormalization, EmpiricalNormalization
from .rnn import RNN, HiddenState

__all__ = [
    "CNN",
    "MLP",
    "RNN",
    "BetaDistribution",
    "Distribution",
    "EmpiricalDiscountedVariationNormalization",
    "EmpiricalNormalization",
    "GaussianDistribution",
    "HeteroscedasticGaussianDistribution",
    "HiddenState",
]
