"""Supervised fine-tuning loop (reference: ``nemo_rl/algorithms/sft.py`` - ``setup`` ``:265``,
``sft_train`` ``:649``; loss ``NLLLossFn`` ``loss_functions.py:1425``).

Batches are message logs (user / assistant turns); loss is masked to the
trained roles (assistant by default), normalised by the global number of
trained tokens; sequences are packed (THD) by the policy worker.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.algorithms.loss.loss_functions import NLLLossFn
from rl_b200.data.llm_message_utils import add_loss_mask_to_message_log, batched_message_log_to_flat_message
from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["sft_train", "build_sft_batch", "sft_validate"]


def build_sft_batch(batch, roles_to_train_on=("assistant",)) -> BatchedDataDict:
    """Message logs -> right-padded rows with the trained roles' tokens masked in.
    Packed Megatron SFT rows (``packed_segments``) contribute one row per packed
    conversation, its tokens and target mask taken as the preprocessor made them."""
    if batch.get("packed_segments") is not None:
        lm = batch.get("loss_multiplier")
        logs, mult = [], []
        for i, segs in enumerate(batch["packed_segments"]):
            for sgm in segs or []:
                logs.append([{"role": "assistant", "token_ids": sgm["token_ids"],
                              "token_loss_mask": sgm["token_loss_mask"].bool()}])
                mult.append(float(lm[i]) if isinstance(lm, torch.Tensor) else 1.0)
        flat, lengths = batched_message_log_to_flat_message(logs)
        return BatchedDataDict({"input_ids": flat["token_ids"], "input_lengths": lengths,
                                "token_mask": flat["token_loss_mask"].float(), "sample_mask": torch.tensor(mult)})
    logs = batch["message_log"]
    add_loss_mask_to_message_log(logs, roles_to_train_on=roles_to_train_on)
    flat, lengths = batched_message_log_to_flat_message(logs)
    lm = batch.get("loss_multiplier")
    return BatchedDataDict({
        "input_ids": flat["token_ids"], "input_lengths": lengths, "token_mask": flat["token_loss_mask"].float(),
        "sample_mask": lm.float() if isinstance(lm, torch.Tensor) else torch.ones(len(logs)),
    })


@torch.no_grad()
def sft_validate(policy, val_dataloader, max_batches: int = 8) -> dict:
    if val_dataloader is None:
        return {}
    losses = []
    for i, batch in enumerate(val_dataloader):
        if i >= max_batches:
            break
        data = build_sft_batch(batch)
        res = policy.train(data, NLLLossFn(), eval_mode=True)
        losses.append(res["loss"])
    return {"val_loss": sum(losses) / max(1, len(losses))}


def sft_train(policy, train_dataloader, master_config: dict, logger=None, checkpointer=None, save_state=None,
              val_dataloader=None, max_steps: Optional[int] = None, step_callback=None) -> dict:
    cfg = master_config.get("sft", {})
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    val_period = int(cfg.get("val_period", 0) or 0)
    gbs = int(master_config["policy"].get("train_global_batch_size", 32))
    local_gbs = max(1, gbs // max(1, policy.ps.dp_size))
    state = dict(save_state or {"current_step": 0, "current_epoch": 0, "total_steps": 0})
    loss_fn = NLLLossFn()
    step = int(state["current_step"])
    for epoch in range(int(state["current_epoch"]), int(cfg.get("max_num_epochs", 1))):
        for batch in train_dataloader:
            if step >= max_steps:
                return state
            data = build_sft_batch(batch)
            res = policy.train(data, loss_fn, gbs=min(local_gbs, data.size))
            step += 1
            state.update(current_step=step, total_steps=state.get("total_steps", 0) + 1)
            metrics = {"loss": res["loss"], "grad_norm": res["grad_norm"], "lr": res["lr"],
                       "num_unmasked_tokens": res.get("num_unmasked_tokens", 0.0)}
            if logger:
                logger.log_metrics(metrics, step, prefix="train")
            if step_callback:
                step_callback(step, metrics)
            if val_dataloader is not None and val_period and step % val_period == 0:
                vm = sft_validate(policy, val_dataloader)
                if logger:
                    logger.log_metrics(vm, step, prefix="validation")
            out_of_time = checkpointer is not None and checkpointer.deadline_reached()
            if checkpointer is not None and (checkpointer.should_save(step) or out_of_time):
                checkpointer.save(policy, state, train_dataloader, metrics, step)
            if out_of_time:  # saved before the wall-clock deadline; stop here
                return state
        state["current_epoch"] = epoch + 1
    return state
