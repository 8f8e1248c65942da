"""Direct preference optimisation and reward-model training loops.

Reference: ``dpo_train`` (``nemo_rl/algorithms/dpo.py:579``, reference logprobs
precomputed by ``add_ref_logprobs_to_data`` ``:361``; loss ``DPOLossFn``
``loss_functions.py:1650``) and ``rm_train`` (``nemo_rl/algorithms/rm.py:486``,
Bradley-Terry loss on a scalar reward head).

Preference batches are ``(prompt, chosen, rejected)`` token triples; they are
laid out as interleaved rows ``[chosen_0, rejected_0, chosen_1, ...]`` with the
loss mask on the response tokens, and trained with ``pair_rows=True`` so that
each pair stays inside one packed micro-batch.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.algorithms.loss.loss_functions import DPOLossFn, MPOLossFn, PreferenceLossFn
from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["preference_batch", "add_ref_logprobs_to_data", "dpo_train", "rm_train"]


def preference_batch(samples: list[dict], pad_id: int = 0) -> BatchedDataDict:
    rows, masks = [], []
    for s in samples:
        p = s["prompt"]
        for resp in (s["chosen"], s["rejected"]):
            ids = torch.cat([p, resp])
            m = torch.cat([torch.zeros(len(p)), torch.ones(len(resp))])
            rows.append(ids)
            masks.append(m)
    S = max(len(r) for r in rows)
    ids = torch.full((len(rows), S), pad_id, dtype=torch.int64)
    tm = torch.zeros(len(rows), S)
    lens = torch.zeros(len(rows), dtype=torch.int64)
    for i, (r, m) in enumerate(zip(rows, masks)):
        ids[i, : len(r)] = r
        tm[i, : len(m)] = m
        lens[i] = len(r)
    return BatchedDataDict({"input_ids": ids, "input_lengths": lens, "token_mask": tm,
                            "sample_mask": torch.ones(len(rows))})


def add_ref_logprobs_to_data(policy, data: BatchedDataDict) -> BatchedDataDict:
    data["reference_policy_logprobs"] = policy.get_reference_policy_logprobs(data)["reference_logprobs"]
    return data


def _collate_pref(batch) -> list[dict]:
    if isinstance(batch, list):
        return batch
    return [dict(prompt=p, chosen=c, rejected=r) for p, c, r in zip(batch["prompt"], batch["chosen"], batch["rejected"])]


def mpo_train(policy, train_dataloader, master_config: dict, **kw) -> dict:
    """MPO = the DPO loop with ``MPOLossFn`` (reference ``nemo_rl/algorithms/mpo.py:217``)."""
    return dpo_train(policy, train_dataloader, {**master_config, "mpo": master_config.get("mpo", {})}, **kw)


def dpo_train(policy, train_dataloader, master_config: dict, logger=None, checkpointer=None, save_state=None,
              max_steps: Optional[int] = None, step_callback=None) -> dict:
    cfg = master_config.get("dpo", master_config.get("mpo", {}))
    loss_cfg = {**cfg, **(master_config.get("loss_fn") or {})}
    loss_fn = MPOLossFn(loss_cfg) if (master_config.get("mpo") is not None or cfg.get("bco_loss_weight")) \
        else DPOLossFn(loss_cfg)
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    state = dict(save_state or {"current_step": 0, "current_epoch": 0})
    step = int(state["current_step"])
    for epoch in range(int(state["current_epoch"]), int(cfg.get("max_num_epochs", 1))):
        for batch in train_dataloader:
            if step >= max_steps:
                return state
            data = add_ref_logprobs_to_data(policy, preference_batch(_collate_pref(batch)))
            res = policy.train(data, loss_fn, gbs=data.size, pair_rows=True)
            if isinstance(loss_fn, MPOLossFn):
                # one EMA update per step from the globally summed BCO rewards
                state["reward_shift"] = loss_fn.update_reward_shift(res.get("bco_reward_sum", 0.0),
                                                                    res.get("bco_reward_count", 0.0))
            step += 1
            state["current_step"] = step
            metrics = {k: res[k] for k in ("loss", "grad_norm", "lr", "accuracy", "preference_loss", "bco_loss")
                       if k in res}
            if logger:
                logger.log_metrics(metrics, step, prefix="train")
            if step_callback:
                step_callback(step, metrics)
            out_of_time = checkpointer is not None and checkpointer.deadline_reached()
            if checkpointer is not None and (checkpointer.should_save(step) or out_of_time):
                checkpointer.save(policy, state, train_dataloader, metrics, step)
            if out_of_time:  # saved before the wall-clock deadline; stop here
                return state
        state["current_epoch"] = epoch + 1
    return state


def rm_train(reward_model, train_dataloader, master_config: dict, logger=None, checkpointer=None, save_state=None,
             max_steps: Optional[int] = None, step_callback=None) -> dict:
    """``reward_model`` is a PolicyWorker built with ``num_labels: 1``."""
    cfg = master_config.get("rm", {})
    loss_fn = PreferenceLossFn()
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    state = dict(save_state or {"current_step": 0, "current_epoch": 0})
    step = int(state["current_step"])
    for epoch in range(int(state["current_epoch"]), int(cfg.get("max_num_epochs", 1))):
        for batch in train_dataloader:
            if step >= max_steps:
                return state
            data = preference_batch(_collate_pref(batch))
            res = reward_model.train(data, loss_fn, gbs=data.size, pair_rows=True)
            step += 1
            state["current_step"] = step
            metrics = {k: res[k] for k in ("loss", "grad_norm", "lr", "accuracy") if k in res}
            if logger:
                logger.log_metrics(metrics, step, prefix="train")
            if step_callback:
                step_callback(step, metrics)
            out_of_time = checkpointer is not None and checkpointer.deadline_reached()
            if checkpointer is not None and (checkpointer.should_save(step) or out_of_time):
                checkpointer.save(reward_model, state, train_dataloader, metrics, step)
            if out_of_time:  # saved before the wall-clock deadline; stop here
                return state
        state["current_epoch"] = epoch + 1
    return state
