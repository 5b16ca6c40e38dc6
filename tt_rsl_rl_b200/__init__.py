"""tt_rsl_rl_b200: on-policy reinforcement learning (rsl_rl's API and checkpoints) built for NVIDIA B200 (sm_100a).

Import paths mirror rsl_rl: ``tt_rsl_rl_b200.runners.OnPolicyRunner``, ``tt_rsl_rl_b200.algorithms.PPO``,
``tt_rsl_rl_b200.models.MLPModel`` and so on. Bare class names in configurations (``"PPO"``, ``"MLPModel"``,
``"GaussianDistribution"``) resolve to this package.
"""

__version__ = "0.1.0"
