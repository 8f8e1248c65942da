"""On-policy distillation (OPD) with one or several teachers (MOPD).

Reference: ``nemo_rl/algorithms/opd.py`` (config block ``on_policy_distillation``,
``resolve_reference_aliases`` ``:336``, ``get_teacher_routing_metrics`` ``:370``,
teacher log-prob enrichment ``:395``) and ``OPDAdvantageEstimator``.  The config
keys and the alias-resolution rules are kept::

    on_policy_distillation:
      enabled: true
      teacher_model_by_agent_name:        # routing alias -> teacher model
        math: llama3.1-8b                 # a model preset name or an HF checkpoint directory
        code: /ckpts/code_teacher
      default_teacher_alias: math         # unmapped routing keys use this alias
      strict_agent_name_match: false      # true: an unmapped key is an error
      deduplicate_shared_teacher_checkpoints: true

Each rollout row is routed by its agent name (``extra_env_info["agent_name"]``)
or, without one, its task name.  Aliases that name the same model share one
teacher (deduplicated).  Teachers are inference-only policy workers colocated
with the student on the same GPUs; per step, every teacher scores the rows
routed to it (one ``get_logprobs`` call over those rows) and the per-token
advantage is the teacher-student log-prob gap of ``OPDAdvantageEstimator``.
The full-vocabulary variant (``on_policy_distillation.full``) is not built:
only the sampled-token estimator is.
"""

from __future__ import annotations

from typing import Any, Callable, Optional

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["is_opd_enabled", "resolve_reference_aliases", "get_teacher_routing_metrics", "routing_keys",
           "TeacherRouter", "build_teacher_router"]


def _opd_cfg(master_config: dict) -> dict:
    return dict((master_config or {}).get("on_policy_distillation") or {})


def is_opd_enabled(master_config: dict) -> bool:
    return bool(_opd_cfg(master_config).get("enabled", False))


def resolve_reference_aliases(agent_refs: list, teacher_model_by_agent_name: dict, default_teacher_alias:
                              Optional[str] = None, strict_agent_name_match: bool = False) -> list[str]:
    """Teacher alias of every routing key: the key itself when it is mapped, else the
    default alias (an error under strict matching or without a default)."""
    out = []
    for ref in agent_refs:
        name = ref if isinstance(ref, str) else ref["name"]
        if name in teacher_model_by_agent_name:
            out.append(name)
        elif strict_agent_name_match:
            raise ValueError(f"no teacher mapped for agent {name!r}; mapped: {sorted(teacher_model_by_agent_name)}")
        elif default_teacher_alias:
            out.append(default_teacher_alias)
        else:
            raise ValueError(f"no teacher mapped for agent {name!r} and no default_teacher_alias")
    return out


def get_teacher_routing_metrics(reference_aliases: list[str], teacher_model_by_agent_name: dict) -> dict:
    """Distinct aliases used, distinct underlying teacher models, and their ratio."""
    aliases = set(reference_aliases)
    models = set()
    for a in aliases:
        if a not in teacher_model_by_agent_name:
            raise KeyError(f"alias {a!r} is not in teacher_model_by_agent_name")
        models.add(teacher_model_by_agent_name[a])
    return {"on_policy_distillation/teacher_alias_unique": float(len(aliases)),
            "on_policy_distillation/teacher_model_unique": float(len(models)),
            "on_policy_distillation/teacher_alias_to_model_compression": float(len(models) / max(len(aliases), 1))}


def routing_keys(batch: BatchedDataDict) -> list[str]:
    """Per-row routing key: the agent name an environment recorded, else the task."""
    n = batch.size
    infos = batch["extra_env_info"] if "extra_env_info" in batch else [None] * n
    tasks = batch["task_name"] if "task_name" in batch else ["default"] * n
    keys = []
    for info, task in zip(infos, tasks):
        name = (info or {}).get("agent_name") if isinstance(info, dict) else None
        keys.append(str(name or task or "default"))
    return keys


class TeacherRouter:
    """Teacher log-probs for a training batch, each row scored by the teacher its
    routing key resolves to.

    ``teachers`` maps a teacher key (the underlying model) to an object with
    ``get_logprobs(BatchedDataDict) -> {"logprobs": [B, S]}`` (a policy worker);
    ``alias_to_teacher`` maps every alias of ``teacher_model_by_agent_name`` to
    its teacher key."""

    def __init__(self, opd_cfg: dict, teachers: dict[str, Any], alias_to_teacher: dict[str, str]):
        self.cfg = dict(opd_cfg)
        self.mapping = dict(self.cfg.get("teacher_model_by_agent_name") or {})
        self.teachers = teachers
        self.alias_to_teacher = alias_to_teacher
        self.last_metrics: dict = {}

    def teacher_logprobs(self, data: BatchedDataDict, keys: list[str]) -> torch.Tensor:
        aliases = resolve_reference_aliases(keys, self.mapping, self.cfg.get("default_teacher_alias"),
                                            bool(self.cfg.get("strict_agent_name_match", False)))
        out = torch.zeros_like(data["input_ids"], dtype=torch.float32)
        by_teacher: dict[str, list[int]] = {}
        for i, a in enumerate(aliases):
            by_teacher.setdefault(self.alias_to_teacher[a], []).append(i)
        for tkey, rows in by_teacher.items():
            sub = data.select_indices(rows)
            lp = self.teachers[tkey].get_logprobs(sub)["logprobs"].to(out.dtype)
            out[rows, :lp.shape[1]] = lp
        m = get_teacher_routing_metrics(aliases, self.mapping)
        m.update({f"on_policy_distillation/rows_{k}": float(len(v)) for k, v in by_teacher.items()})
        self.last_metrics = m
        return out

    def teacher_topk(self, data: BatchedDataDict, keys: list[str], k: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Each row's top-``k`` next-token log-probs / ids ``[B, S, k]`` from its
        routed teacher (``k`` = vocabulary size: the full distribution)."""
        from rl_b200.algorithms.distillation import teacher_topk

        aliases = resolve_reference_aliases(keys, self.mapping, self.cfg.get("default_teacher_alias"),
                                            bool(self.cfg.get("strict_agent_name_match", False)))
        B, S = data["input_ids"].shape
        vals = torch.zeros(B, S, k, dtype=torch.float32)
        idx = torch.zeros(B, S, k, dtype=torch.int64)
        by_teacher: dict[str, list[int]] = {}
        for i, a in enumerate(aliases):
            by_teacher.setdefault(self.alias_to_teacher[a], []).append(i)
        for tkey, rows in by_teacher.items():
            v, ix = teacher_topk(self.teachers[tkey], data.select_indices(rows), k)
            vals[rows, :v.shape[1]] = v
            idx[rows, :ix.shape[1]] = ix
        self.last_metrics = get_teacher_routing_metrics(aliases, self.mapping)
        return vals, idx


def get_opd_full_config(master_config: dict) -> Optional[dict]:
    """The ``on_policy_distillation.full`` block when enabled (full-vocabulary
    MOPD, the reference's ``opd_full``: an exact reverse KL between the student's
    and the routed teacher's next-token distributions instead of the sampled-token
    gap); None otherwise.  The ``logits`` payload is built here: the teacher's
    log-probabilities over the whole vocabulary (``top_k`` may cap it, default the
    vocabulary size) feed the reverse-KL distillation loss."""
    full = (_opd_cfg(master_config).get("full") or {})
    if not full.get("enabled", False):
        return None
    payload = str(full.get("teacher_payload", "logits"))
    if payload != "logits":
        raise NotImplementedError(f"on_policy_distillation.full.teacher_payload {payload!r}: only 'logits' is built")
    if str(full.get("divergence", "reverse_kl")) != "reverse_kl":
        raise ValueError("on_policy_distillation.full.divergence must be reverse_kl")
    return dict(full)


def build_teacher_router(master_config: dict, student, make_teacher: Optional[Callable[[str], Any]] = None
                         ) -> TeacherRouter:
    """Create one inference-only teacher per distinct model of
    ``teacher_model_by_agent_name`` (per alias when deduplication is off).
    ``make_teacher(model_ref)`` overrides how a teacher is built; by default it is
    a policy worker on the student's parallel layout whose weights come from the
    HF checkpoint directory ``model_ref`` or, for a preset name, its random init
    (offline runs)."""
    cfg = _opd_cfg(master_config)
    mapping = dict(cfg.get("teacher_model_by_agent_name") or {})
    if not mapping:
        raise ValueError("on_policy_distillation.teacher_model_by_agent_name is empty")
    dedup = bool(cfg.get("deduplicate_shared_teacher_checkpoints", True))
    alias_to_teacher = {a: (m if dedup else f"{a}:{m}") for a, m in mapping.items()}
    make_teacher = make_teacher or (lambda ref: _default_teacher(master_config, student, ref))
    teachers = {}
    for a, m in mapping.items():
        key = alias_to_teacher[a]
        if key not in teachers:
            teachers[key] = make_teacher(m)
    return TeacherRouter(cfg, teachers, alias_to_teacher)


def _default_teacher(master_config: dict, student, model_ref: str):
    import os

    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker

    pcfg = dict(master_config["policy"])
    mcfg = get_model_config(model_ref)
    t = PolicyWorker(pcfg, model_cfg=mcfg, pstate=student.ps, seed=int(master_config.get("grpo", {}).get("seed", 0))
                     + 1000, init_reference_model=False)
    if os.path.isdir(model_ref):
        t.load_checkpoint(model_ref)
    return t
