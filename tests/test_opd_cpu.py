"""On-policy distillation with routed teachers (MOPD): alias resolution, routing
metrics, per-row teacher scoring with shared teachers, and a tiny GRPO run whose
student moves toward its teacher (CPU)."""

from __future__ import annotations

import pytest
import torch

from rl_b200.algorithms.opd import (TeacherRouter, build_teacher_router, get_teacher_routing_metrics,
                                    resolve_reference_aliases, routing_keys)
from rl_b200.distributed.batched_data_dict import BatchedDataDict


def test_alias_resolution_rules():
    mapping = {"math": "m1", "code": "m2"}
    assert resolve_reference_aliases(["math", "code", "chat"], mapping, "math") == ["math", "code", "math"]
    assert resolve_reference_aliases([{"name": "code"}], mapping) == ["code"]
    with pytest.raises(ValueError):
        resolve_reference_aliases(["chat"], mapping, "math", strict_agent_name_match=True)
    with pytest.raises(ValueError):
        resolve_reference_aliases(["chat"], mapping)
    m = get_teacher_routing_metrics(["a", "b", "a"], {"a": "x", "b": "x"})
    assert m["on_policy_distillation/teacher_alias_unique"] == 2.0
    assert m["on_policy_distillation/teacher_model_unique"] == 1.0
    assert m["on_policy_distillation/teacher_alias_to_model_compression"] == 0.5


class _FakeTeacher:
    def __init__(self, value):
        self.value, self.calls = value, []

    def get_logprobs(self, data):
        self.calls.append(data.size)
        return {"logprobs": torch.full(data["input_ids"].shape, float(self.value))}


def test_router_scores_each_row_with_its_teacher_once_per_model():
    cfg = {"teacher_model_by_agent_name": {"math": "M", "algebra": "M", "code": "C"},
           "default_teacher_alias": "code"}
    made = {}

    def make(ref):
        made[ref] = _FakeTeacher({"M": -1.0, "C": -2.0}[ref])
        return made[ref]

    router = build_teacher_router({"on_policy_distillation": cfg}, student=None, make_teacher=make)
    assert sorted(made) == ["C", "M"]  # "math" and "algebra" share one teacher
    data = BatchedDataDict({"input_ids": torch.zeros(5, 3, dtype=torch.long),
                            "task_name": ["math", "code", "algebra", "chat", "math"],
                            "extra_env_info": [None, None, None, {"agent_name": "math"}, None]})
    keys = routing_keys(data)
    assert keys == ["math", "code", "algebra", "math", "math"]
    lp = router.teacher_logprobs(data, keys)
    assert lp[:, 0].tolist() == [-1.0, -2.0, -1.0, -1.0, -1.0]
    assert made["M"].calls == [4] and made["C"].calls == [1]
    assert router.last_metrics["on_policy_distillation/teacher_model_unique"] == 2.0


def test_grpo_on_policy_distillation_trains_on_teacher_student_gap():
    """End to end through grpo_train: every step's training batch carries the
    routed teacher's log-probs and advantages equal to the per-token teacher -
    student gap on generated tokens (the student's log-probs taken before the
    update), and the update runs on them."""
    from rl_b200.algorithms.grpo import grpo_train
    from rl_b200.data.datasets import StatefulDataLoader, SyntheticPromptDataset
    from rl_b200.environments.synthetic import EvenTokenEnvironment
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker

    mcfg = get_model_config("tiny-llama")
    pcfg = {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 16,
            "optimizer": {"kwargs": {"lr": 1e-3, "weight_decay": 0.0}},
            "generation": {"temperature": 1.0, "max_new_tokens": 8},
            "sequence_packing": {"train_mb_tokens": 256, "logprob_mb_tokens": 256}}
    student = PolicyWorker(pcfg, model_cfg=mcfg, seed=0)
    teacher = PolicyWorker(pcfg, model_cfg=mcfg, seed=7, init_reference_model=False)
    with torch.no_grad():  # a teacher with a sharper distribution than the random student
        teacher.model.param("lm_head.weight").mul_(5.0)
    opd = {"enabled": True, "teacher_model_by_agent_name": {"synthetic": "tiny-llama"}}
    router = TeacherRouter(opd, {"tiny-llama": teacher}, {"synthetic": "tiny-llama"})
    cfg = {"grpo": {"num_prompts_per_step": 4, "num_generations_per_prompt": 4, "max_num_steps": 2, "seed": 0},
           "loss_fn": {"reference_policy_kl_penalty": 0.0}, "policy": pcfg, "on_policy_distillation": opd}
    seen = []
    real_train = student.train

    def spy(data, loss_fn, **kw):
        before = student.get_logprobs(data)["logprobs"]
        out = real_train(data, loss_fn, **kw)
        seen.append((data, before, out))
        return out

    student.train = spy
    dl = StatefulDataLoader(SyntheticPromptDataset(64, 8, 8, mcfg.vocab_size, seed=1), 4, shuffle=False)
    metrics = []
    grpo_train(student, dl, {"synthetic": EvenTokenEnvironment({})}, cfg, teacher_router=router,
               step_callback=lambda s, m: metrics.append(m))
    assert len(seen) == 2 and len(metrics) == 2
    for data, before, out in seen:
        tm = data["token_mask"]
        tlp = teacher.get_logprobs(data)["logprobs"]
        torch.testing.assert_close(data["teacher_logprobs"], tlp)
        torch.testing.assert_close(data["prev_logprobs"] * tm, before * tm, atol=1e-5, rtol=0)
        torch.testing.assert_close(data["advantages"], (tlp - before) * tm, atol=1e-5, rtol=0)
        assert tm.sum() > 0 and out["grad_norm"] > 0
    gap = metrics[0]["on_policy_distillation/teacher_student_logprob_gap_mean"]
    assert gap < 0 and metrics[0]["on_policy_distillation/teacher_model_unique"] == 1.0


def test_full_vocabulary_opd_reverse_kl():
    """``on_policy_distillation.full``: each step trains on the exact reverse KL
    between the student's and the routed teacher's full next-token
    distributions; the loss equals that KL computed by hand on the batch, and
    training lowers it."""
    from rl_b200.algorithms.grpo import grpo_train
    from rl_b200.algorithms.loss.loss_functions import DistillationLossFn
    from rl_b200.data.datasets import StatefulDataLoader, SyntheticPromptDataset
    from rl_b200.environments.synthetic import EvenTokenEnvironment
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker

    mcfg = get_model_config("tiny-llama")
    pcfg = {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 16,
            "optimizer": {"kwargs": {"lr": 3e-3, "weight_decay": 0.0}},
            "generation": {"temperature": 1.0, "max_new_tokens": 8},
            "sequence_packing": {"train_mb_tokens": 256, "logprob_mb_tokens": 256}}
    student = PolicyWorker(pcfg, model_cfg=mcfg, seed=0)
    teacher = PolicyWorker(pcfg, model_cfg=mcfg, seed=7, init_reference_model=False)
    opd = {"enabled": True, "teacher_model_by_agent_name": {"synthetic": "tiny-llama"}, "full": {"enabled": True}}
    router = TeacherRouter(opd, {"tiny-llama": teacher}, {"synthetic": "tiny-llama"})
    cfg = {"grpo": {"num_prompts_per_step": 4, "num_generations_per_prompt": 4, "max_num_steps": 4, "seed": 0},
           "loss_fn": {"reference_policy_kl_penalty": 0.0}, "policy": pcfg, "on_policy_distillation": opd}
    seen = []
    real_train = student.train

    def spy(data, loss_fn, **kw):
        seen.append((data, loss_fn))
        return real_train(data, loss_fn, **kw)

    student.train = spy
    dl = StatefulDataLoader(SyntheticPromptDataset(64, 8, 8, mcfg.vocab_size, seed=1), 4, shuffle=False)
    metrics = []
    grpo_train(student, dl, {"synthetic": EvenTokenEnvironment({})}, cfg, teacher_router=router,
               step_callback=lambda s, m: metrics.append(m))
    data, lf = seen[0]
    assert isinstance(lf, DistillationLossFn) and lf.kl_type == "reverse"
    assert data["teacher_topk_logprobs"].shape[-1] == mcfg.vocab_size  # the whole distribution
    # the teacher payload is the teacher's full log-softmax
    p = data["teacher_topk_logprobs"][0, 1:3].exp().sum(-1)
    torch.testing.assert_close(p, torch.ones_like(p), atol=1e-4, rtol=0)
    losses = [m["loss"] for m in metrics]
    assert losses[-1] < losses[0], losses
