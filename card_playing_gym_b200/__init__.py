"""B200-native self-play hot path of card_playing_gym (rollout decode + PPO advantage/loss).

Python/PyTorch host code over a C-ABI CUDA library (``libcg_b200.so``, sm_100a) built
in-tree by ``python -m card_playing_gym_b200.build``. There is no CPU fallback: every
entry point raises if the library is missing or a tensor is not on a CUDA device.
"""

from .config import RL_V6, SMOKE, PlumpModelConfig, TrunkConfig, synthetic_plump_actor_state

__all__ = ["RL_V6", "SMOKE", "PlumpModelConfig", "TrunkConfig", "synthetic_plump_actor_state"]
