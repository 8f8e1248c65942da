"""Knowledge distillation loops.

* ``distillation_train`` - on-policy distillation (reference: ``nemo_rl/algorithms/opd.py``
  ``OnPolicyDistillationConfig`` ``:158``, MOPD): the student generates, the teacher
  scores the sampled tokens, and the per-token advantage is the (proximal)
  teacher log-probability minus the student's (``OPDAdvantageEstimator``); the
  student is updated with the clipped policy-gradient loss.  Teacher and student
  only exchange ``[B, S]`` log-probabilities - no vocabulary-sized tensors.
* ``kd_train`` - off-policy top-k logit distillation on fixed data (reference:
  ``distillation_train`` ``nemo_rl/algorithms/distillation.py:1251`` with
  ``DistillationLossFn``): the teacher's top-k next-token distribution is
  matched by the student (forward / reverse / mixed KL).
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.algorithms.advantage_estimator import OPDAdvantageEstimator
from rl_b200.algorithms.grpo import build_train_data
from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn, DistillationLossFn
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.experience.rollouts import run_multi_turn_rollout

__all__ = ["distillation_train", "kd_train", "teacher_topk"]


class _Zero:
    def compute_advantage(self, prompt_ids, rewards, mask, **kw):
        return torch.zeros_like(mask)


def distillation_train(student, teacher, dataloader, task_to_env: dict, master_config: dict, logger=None,
                       max_steps: Optional[int] = None, step_callback=None, tokenizer=None) -> dict:
    cfg = master_config.get("distillation", {})
    loss_cfg = dict(master_config.get("loss_fn", {}))
    loss = ClippedPGLossFn(loss_cfg)
    est = OPDAdvantageEstimator(cfg.get("adv_estimator", {}))
    G = int(cfg.get("num_generations_per_prompt", 1))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    step = 0
    for batch in dataloader:
        if step >= max_steps:
            break
        rep = batch.repeat_interleave(G)
        rep["group_id"] = torch.arange(len(batch["message_log"])).repeat_interleave(G)
        student.prepare_for_generation(len(rep["message_log"]))
        rollout, _ = run_multi_turn_rollout(student, rep, tokenizer, task_to_env, max_seq, 1)
        student.finish_generation()
        data, _ = build_train_data(rollout, _Zero(), {}, loss_cfg, rollout["group_id"])
        data["prev_logprobs"] = student.get_logprobs(data)["logprobs"]
        t_lp = teacher.get_logprobs(data)["logprobs"]
        adv = est.compute_advantage(None, None, data["token_mask"], logprobs_policy=data["prev_logprobs"],
                                    logprobs_teacher=t_lp)
        data["advantages"] = adv
        res = student.train(data, loss)
        student.refit()
        step += 1
        mask = data["token_mask"]
        rev_kl = float(((data["prev_logprobs"] - t_lp) * mask).sum() / mask.sum().clamp_min(1))
        metrics = {"loss": res["loss"], "grad_norm": res["grad_norm"], "reverse_kl_sampled": rev_kl}
        if logger:
            logger.log_metrics(metrics, step, prefix="train")
        if step_callback:
            step_callback(step, metrics)
    return {"current_step": step}


@torch.no_grad()
def teacher_topk(teacher, data: BatchedDataDict, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Teacher top-k next-token log-probs and ids, ``[B, S, k]`` aligned so that
    position i holds the distribution of token i (position 0 unused)."""
    from rl_b200.algorithms.loss.interfaces import LossInputType

    class _Logit:
        input_type = LossInputType.LOGIT

    ids = data["input_ids"]
    B, S = ids.shape
    lengths = [int(x) for x in data["input_lengths"].tolist()]
    vals = torch.zeros(B, S, k)
    idx = torch.zeros(B, S, k, dtype=torch.int64)
    for b in range(B):
        width = lengths[b]
        logits = teacher._loss_input(_Logit(), ids, lengths, [b], width, 1.0)[0]   # [width-1, V]
        lp = torch.log_softmax(logits.float(), -1)
        v, i = lp.topk(k, dim=-1)
        vals[b, 1:width] = v.cpu()
        idx[b, 1:width] = i.cpu()
    return vals, idx


def kd_train(student, teacher, batches, master_config: dict, k: int = 16, max_steps: Optional[int] = None,
             step_callback=None) -> dict:
    """``batches``: iterable of BatchedDataDicts with input_ids / input_lengths /
    token_mask / sample_mask (e.g. SFT data)."""
    cfg = master_config.get("distillation", {})
    loss = DistillationLossFn(cfg.get("loss_fn", {}))
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    step = 0
    for data in batches:
        if step >= max_steps:
            break
        v, i = teacher_topk(teacher, data, k)
        data["teacher_topk_logprobs"], data["teacher_topk_indices"] = v, i
        res = student.train(data, loss)
        step += 1
        if step_callback:
            step_callback(step, {"loss": res["loss"], "grad_norm": res["grad_norm"]})
    return {"current_step": step}
