"""Evaluation datasets: benchmark rows rekeyed for the math and multiple-choice
processors, each with its task spec and processor bound.

Reference: ``nemo_rl/data/datasets/eval_datasets/__init__.py`` (``load_eval_dataset``:
``mmlu`` / ``mmlu_<LANG>``, ``mmlu_pro``, ``gpqa`` / ``gpqa_diamond``, ``math`` /
``math500``, any other name a local CSV / JSON file), ``math.py``, ``gpqa.py``,
``mmlu.py``, ``mmlu_pro.py``, ``local_math_dataset.py``.  The names, the rekeyed
row fields (``problem`` / ``expected_answer``; ``question`` / ``options`` /
``answer`` / ``subject``) and the task names are kept, so eval configs written for
the reference select the same rows here.

Offline: each dataset takes ``data_path``, a local copy of the benchmark's raw
file (the simple-evals CSVs, the hub parquet / jsonl); without it the source is
read through ``datasets.load_dataset``, which in a container with no network
resolves only from the local cache.  The audio / video benchmarks (MMAU,
Daily-Omni) are not built.

Design difference: GPQA shuffles each question's four choices with a seeded
generator (``seed``, default 0), so an evaluation is reproducible; the reference
draws them from an unseeded one.
"""

from __future__ import annotations

import os
import random
from typing import Optional

from rl_b200.data.processors import TaskDataSpec, math_data_processor, multichoice_qa_processor
from rl_b200.data.response_datasets import Rows, load_rows

__all__ = ["MathDataset", "GPQADataset", "MMLUDataset", "MMLUProDataset", "LocalMathDataset", "MMLU_LANGUAGES",
           "load_eval_dataset", "setup_eval_data"]

SIMPLE_EVALS = "https://openaipublic.blob.core.windows.net/simple-evals"
MMLU_LANGUAGES = ("AR-XY", "BN-BD", "DE-DE", "EN-US", "ES-LA", "FR-FR", "HI-IN", "ID-ID", "IT-IT", "JA-JP", "KO-KR",
                  "PT-BR", "ZH-CN", "SW-KE", "YO-NG")


def _csv_rows(url: str, data_path: Optional[str]) -> Rows:
    if data_path:
        return load_rows(data_path, None, None)
    import datasets

    try:
        return Rows(datasets.load_dataset("csv", data_files=url, split="train"))
    except Exception as e:  # noqa: BLE001 - say what to do offline
        raise RuntimeError(f"could not read {url} ({type(e).__name__}); pass data_path pointing at a local copy") from e


def _hub_rows(hub: str, subset: Optional[str], split: str, data_path: Optional[str]) -> Rows:
    return load_rows(data_path, None, None) if data_path else load_rows(hub, subset, split)


class _EvalDataset:
    rekeyed_ds: Rows
    task_spec: TaskDataSpec
    processor = None

    def _bind(self, task_name: str, prompt_file: Optional[str], system_prompt_file: Optional[str], processor):
        self.task_spec = TaskDataSpec(task_name=task_name, prompt_file=prompt_file,
                                      system_prompt_file=system_prompt_file)
        self.processor = processor

    def __len__(self) -> int:
        return len(self.rekeyed_ds)


class MathDataset(_EvalDataset):
    """MATH test sets of simple-evals (``math_test`` or ``math_500_test`` CSV:
    ``Question`` / ``Answer``)."""

    def __init__(self, variant: str = "math_test", prompt_file: Optional[str] = None,
                 system_prompt_file: Optional[str] = None, data_path: Optional[str] = None):
        if variant not in ("math_test", "math_500_test"):
            raise ValueError(f"MATH variant must be math_test or math_500_test, not {variant!r}")
        self.rekeyed_ds = _csv_rows(f"{SIMPLE_EVALS}/{variant}.csv", data_path).map(
            lambda r: {"problem": r["Question"], "expected_answer": r["Answer"]})
        self._bind(variant, prompt_file, system_prompt_file, math_data_processor)


class GPQADataset(_EvalDataset):
    """GPQA (``main`` or ``diamond``): the correct and three incorrect answers
    shuffled into options A-D (seeded per row), ``answer`` the correct letter."""

    def __init__(self, variant: str = "diamond", prompt_file: Optional[str] = None,
                 system_prompt_file: Optional[str] = None, data_path: Optional[str] = None, seed: int = 0):
        if variant not in ("diamond", "main"):
            raise ValueError(f"GPQA variant must be diamond or main, not {variant!r}")
        self.seed = int(seed)
        base = _hub_rows("Idavidrein/gpqa", f"gpqa_{variant}", "train", data_path)
        self.rekeyed_ds = Rows([self._rekey(i, base.raw(i)) for i in range(len(base))])
        self._bind(f"GPQA_{variant}", prompt_file, system_prompt_file, multichoice_qa_processor)

    def _rekey(self, i: int, row: dict) -> dict:
        choices = [row["Correct Answer"], row["Incorrect Answer 1"], row["Incorrect Answer 2"],
                   row["Incorrect Answer 3"]]
        order = random.Random(self.seed * 1_000_003 + i).sample(range(4), 4)
        choices = [choices[j] for j in order]
        return {"question": row["Question"], "options": dict(zip("ABCD", choices)),
                "answer": "ABCD"[choices.index(row["Correct Answer"])]}


class MMLUDataset(_EvalDataset):
    """MMLU (English) or one of simple-evals' translated sets: ``Question``,
    ``A``-``D``, ``Answer``, ``Subject``."""

    def __init__(self, language: str = "EN-US", prompt_file: Optional[str] = None,
                 system_prompt_file: Optional[str] = None, data_path: Optional[str] = None):
        if language not in MMLU_LANGUAGES:
            raise ValueError(f"MMLU language must be one of {MMLU_LANGUAGES}, not {language!r}")
        name = "mmlu.csv" if language == "EN-US" else f"mmlu_{language}.csv"
        self.rekeyed_ds = _csv_rows(f"{SIMPLE_EVALS}/{name}", data_path).map(
            lambda r: {"question": r["Question"], "options": {k: r[k] for k in "ABCD"}, "answer": r["Answer"],
                       "subject": r["Subject"]})
        self._bind(f"MMLU_{language}", prompt_file, system_prompt_file, multichoice_qa_processor)


class MMLUProDataset(_EvalDataset):
    """MMLU-Pro test split: up to ten options lettered from A, ``category`` as the
    subject."""

    def __init__(self, prompt_file: Optional[str] = None, system_prompt_file: Optional[str] = None,
                 data_path: Optional[str] = None):
        self.rekeyed_ds = _hub_rows("TIGER-Lab/MMLU-Pro", None, "test", data_path).map(
            lambda r: {"question": r["question"], "options": {chr(65 + i): o for i, o in enumerate(r["options"])},
                       "answer": r["answer"], "subject": r["category"]})
        self._bind("MMLU-Pro", prompt_file, system_prompt_file, multichoice_qa_processor)


class LocalMathDataset(_EvalDataset):
    """A local CSV / JSON math set: ``problem_key`` and ``solution_key`` columns;
    task name = the file's base name."""

    def __init__(self, data_path: str, problem_key: str, solution_key: str, split: Optional[str] = None,
                 file_format: str = "csv", prompt_file: Optional[str] = None,
                 system_prompt_file: Optional[str] = None):
        if file_format not in ("csv", "json"):
            raise ValueError(f"file_format must be csv or json, not {file_format!r}")
        rows = load_rows(data_path, None, split if not os.path.isfile(data_path) else None)
        self.rekeyed_ds = rows.map(lambda r: {"problem": r[problem_key], "expected_answer": r[solution_key]})
        self._bind(os.path.basename(data_path).split(".")[0], prompt_file, system_prompt_file, math_data_processor)


def load_eval_dataset(data_config: dict) -> _EvalDataset:
    """The evaluation dataset ``data_config["dataset_name"]`` names (see the module
    docstring); ``prompt_file`` / ``system_prompt_file`` / ``data_path`` pass through."""
    name = data_config["dataset_name"]
    common = {"prompt_file": data_config.get("prompt_file"),
              "system_prompt_file": data_config.get("system_prompt_file")}
    dp = data_config.get("data_path")
    if name == "mmlu":
        return MMLUDataset(data_path=dp, **common)
    if name.startswith("mmlu_") and name != "mmlu_pro":
        return MMLUDataset(language=name.split("_", 1)[1], data_path=dp, **common)
    if name == "mmlu_pro":
        return MMLUProDataset(data_path=dp, **common)
    if name in ("gpqa", "gpqa_diamond"):
        return GPQADataset(variant="main" if name == "gpqa" else "diamond", data_path=dp,
                           seed=int(data_config.get("seed", 0)), **common)
    if name in ("math", "math500"):
        return MathDataset(variant="math_test" if name == "math" else "math_500_test", data_path=dp, **common)
    if name in ("mmau", "TwinkStart/MMAU", "daily-omni"):
        raise NotImplementedError(f"{name!r} is an audio / video benchmark; multimodal evaluation is not built")
    return LocalMathDataset(data_path=name, problem_key=data_config["problem_key"],
                            solution_key=data_config["solution_key"], split=data_config.get("split"),
                            file_format=data_config.get("file_format", "csv"), **common)


def setup_eval_data(tokenizer, data_config: dict):
    """``(processed dataset, eval dataset)`` for an ``eval`` run: the benchmark's
    rows through its processor at ``data_config["max_input_seq_length"]``, ready
    for a ``StatefulDataLoader`` and ``run_env_eval`` (reference:
    ``examples/run_eval.py`` ``setup_data``)."""
    from rl_b200.data.utils import AllTaskProcessedDataset

    base = load_eval_dataset(data_config)
    ds = AllTaskProcessedDataset(base.rekeyed_ds, tokenizer, base.task_spec, base.processor,
                                 max_seq_length=data_config.get("max_input_seq_length"))
    return ds, base
