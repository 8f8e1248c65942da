"""Evaluation (pass@k / cons@k over environment rewards)."""

from rl_b200.evals.eval import eval_cons_k, eval_pass_k, run_env_eval

__all__ = ["eval_pass_k", "eval_cons_k", "run_env_eval"]
