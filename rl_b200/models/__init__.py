"""rl_b200 subpackage."""
