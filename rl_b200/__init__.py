"""rl_b200: a Blackwell-native (sm_100a) RL post-training framework.

GRPO / DAPO / PPO / SFT / DPO loops over a PyTorch model whose hot ops are
hand-written sm_100a CUDA kernels (``csrc/``, built in-tree into ``rl_b200._C``).
"""

__version__ = "0.1.0"
