"""Data + environment set-up from the ``data:`` / ``env:`` config blocks.

Reference: ``nemo_rl/data/utils.py:152`` (``setup_response_data``),
``nemo_rl/data/datasets/processed_dataset.py`` (``AllTaskProcessedDataset``)
and ``nemo_rl/data/datasets/utils.py`` (``update_single_dataset_config``,
``merge_datasets``, ``extract_necessary_env_names``).  The config schema is the
reference's::

    data:
      max_input_seq_length: 1024
      shuffle: true
      default:                     # filled into every train / validation entry
        prompt_file: ...
        processor: math_hf_data_processor
        env_name: math
      train:                       # one entry or a list
        dataset_name: OpenMathInstruct-2      # or ResponseDataset + data_path, ...
        split_validation_size: 0.05
      validation:
        dataset_name: AIME2024
    env:
      math: {num_workers: 8}

Each dataset is bound to its processor and task spec by task name; the merged
training set formats and tokenises rows on access.
"""

from __future__ import annotations

import copy
from typing import Any, Callable, Optional

from rl_b200.data.processors import TaskDataSpec
from rl_b200.data.response_datasets import Rows, load_response_dataset

__all__ = ["AllTaskProcessedDataset", "setup_response_data", "merge_datasets", "extract_necessary_env_names",
           "update_single_dataset_config", "create_env"]


class AllTaskProcessedDataset:
    """Formatted rows -> ``DatumSpec`` through the processor of each row's task.

    ``task_data_processors`` is one processor (single task, with
    ``default_task_data_spec``) or ``{task_name: (TaskDataSpec, processor)}``; task
    specs without a prompt / system prompt take the default spec's."""

    def __init__(self, dataset, tokenizer, default_task_data_spec: Optional[TaskDataSpec],
                 task_data_processors: dict | Callable, task_data_preprocessors: dict | Callable | None = None,
                 max_seq_length: Optional[int] = None):
        self.dataset = dataset
        self.tokenizer = tokenizer
        self.default_task_data_spec = default_task_data_spec
        self.task_data_processors = task_data_processors
        self.task_data_preprocessors = task_data_preprocessors
        self.max_seq_length = max_seq_length
        if isinstance(task_data_processors, dict) and default_task_data_spec is not None:
            for spec, _ in task_data_processors.values():
                spec.copy_defaults(default_task_data_spec)

    def __len__(self) -> int:
        return len(self.dataset)

    def __getitem__(self, idx: int) -> dict:
        row = self.dataset[idx]
        pre = self.task_data_preprocessors
        if isinstance(pre, dict):
            pre = pre.get(row.get("task_name"))
        if pre is not None:
            row = pre(row)
        if isinstance(self.task_data_processors, dict):
            task = row.get("task_name")
            if task not in self.task_data_processors:
                raise KeyError(f"no processor bound to task {task!r}; bound: {sorted(self.task_data_processors)}")
            spec, proc = self.task_data_processors[task]
        else:
            spec, proc = self.default_task_data_spec, self.task_data_processors
        datum = proc(row, spec, self.tokenizer, self.max_seq_length, idx)
        datum.setdefault("task_name", row.get("task_name", "default"))
        return datum


class _Concat:
    def __init__(self, parts):
        self.parts = list(parts)
        self.offsets = []
        n = 0
        for p in self.parts:
            self.offsets.append(n)
            n += len(p)
        self.n = n

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        if i < 0:
            i += self.n
        for p, off in zip(reversed(self.parts), reversed(self.offsets)):
            if i >= off:
                return p[i - off]
        raise IndexError(i)


def merge_datasets(datasets: list) -> Any:
    """One indexable dataset over several (concatenated in order)."""
    if not datasets:
        raise ValueError("no datasets to merge")
    return datasets[0] if len(datasets) == 1 else Rows(_Concat(datasets))


def update_single_dataset_config(data_config: dict, default: dict) -> None:
    """Fill keys missing from one dataset entry with the ``default`` entry's."""
    for k, v in (default or {}).items():
        data_config.setdefault(k, copy.deepcopy(v))


def extract_necessary_env_names(data_config: dict) -> list[str]:
    """Environment names referenced by the train / validation / default entries."""
    names = []
    for key in ("train", "validation", "default"):
        entries = data_config.get(key)
        for e in (entries if isinstance(entries, list) else [entries]):
            if isinstance(e, dict) and e.get("env_name") and e["env_name"] not in names:
                names.append(e["env_name"])
    return names


def create_env(env_name: str, env_config: Optional[dict], tokenizer=None):
    """Environment ``env_name`` (or ``env_config["kind"]``) from the registry; the
    tokenizer's ``decode`` turns generated ids into text for verifiers."""
    from rl_b200.environments.registry import make_environment

    cfg = dict(env_config or {})
    kind = cfg.get("kind", env_name)
    decode = getattr(tokenizer, "decode", None)
    if decode is not None:
        try:
            return make_environment(kind, cfg, decode=decode)
        except TypeError:
            pass
    return make_environment(kind, cfg)


def _entries(x) -> list[dict]:
    if x is None:
        return []
    return [x] if isinstance(x, dict) else list(x)


def setup_response_data(tokenizer, data_config: dict, env_configs: Optional[dict] = None, is_vlm: bool = False,
                        *, load_validation: bool = True, context_parallel_size: Optional[int] = None):
    """Train / validation datasets (and, with ``env_configs``, the task -> environment
    maps) from the ``data:`` block (``context_parallel_size``: the policy's, for
    packed Megatron SFT data).  Returns ``(train, val)`` without environment
    configs, else ``(train, val, task_to_env, val_task_to_env)``; ``val`` is None
    when no validation data is configured."""
    if is_vlm:
        raise NotImplementedError("vision-language data processing is not part of this framework")
    data_config = copy.deepcopy(data_config)
    default = data_config.get("default") or {}
    max_len = data_config.get("max_input_seq_length")
    envs = {}
    if env_configs is not None:
        for name in extract_necessary_env_names(data_config):
            envs[name] = create_env(name, env_configs.get(name), tokenizer)

    procs, pres, task_to_env, parts = {}, {}, {}, []
    val_procs, val_pres, val_task_to_env, val_parts = {}, {}, {}, []
    for cfg in _entries(data_config.get("train")):
        update_single_dataset_config(cfg, default)
        ds = load_response_dataset(cfg, context_parallel_size=context_parallel_size)
        parts.append(ds.dataset)
        procs[ds.task_name] = (ds.task_spec, ds.processor)
        if ds.preprocessor is not None:
            pres[ds.task_name] = ds.preprocessor
        if env_configs is not None and cfg.get("env_name"):
            task_to_env[ds.task_name] = envs[cfg["env_name"]]
        if load_validation and ds.val_dataset is not None:
            val_parts.append(ds.val_dataset)
            val_procs[ds.task_name] = procs[ds.task_name]
            if ds.task_name in pres:
                val_pres[ds.task_name] = pres[ds.task_name]
            if ds.task_name in task_to_env:
                val_task_to_env[ds.task_name] = task_to_env[ds.task_name]
    if not parts:
        raise ValueError("data.train names no dataset")
    if load_validation:
        for cfg in _entries(data_config.get("validation")):
            update_single_dataset_config(cfg, default)
            ds = load_response_dataset(cfg, context_parallel_size=context_parallel_size)
            val_parts.append(ds.dataset)
            val_procs[ds.task_name] = (ds.task_spec, ds.processor)
            if ds.preprocessor is not None:
                val_pres[ds.task_name] = ds.preprocessor
            if env_configs is not None and cfg.get("env_name"):
                val_task_to_env[ds.task_name] = envs[cfg["env_name"]]
    default_spec = TaskDataSpec(task_name=None, prompt_file=default.get("prompt_file"),
                                system_prompt_file=default.get("system_prompt_file"))
    train = AllTaskProcessedDataset(merge_datasets(parts), tokenizer, default_spec, procs, pres or None, max_len)
    val = (AllTaskProcessedDataset(merge_datasets(val_parts), tokenizer, default_spec, val_procs, val_pres or None,
                                   max_len) if val_parts else None)
    if env_configs is None:
        return train, val
    return train, val, task_to_env, val_task_to_env
