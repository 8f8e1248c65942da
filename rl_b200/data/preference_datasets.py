"""Preference datasets for DPO / reward-model training: rows
``{"context": [turns], "completions": [{"rank", "completion": [turns]}] x 2,
"task_name"}`` (lower rank preferred), turned into chosen / rejected message logs
by ``preference_preprocessor``.

Reference: ``nemo_rl/data/datasets/preference_datasets/__init__.py``
(``DATASET_REGISTRY``, ``load_preference_dataset``), ``binary_preference_dataset.py``,
``preference_dataset.py``, ``helpsteer3.py``, ``tulu3.py``.  Registry names, the
constructor keywords and the row format are kept.  The image-text MMPR
preference set is not built.
"""

from __future__ import annotations

import json
import warnings
from typing import Callable, Optional

from rl_b200.data.processors import preference_preprocessor
from rl_b200.data.response_datasets import (RawDataset, _external_class, _HubResponseDataset, _task_name_of_path,
                                            load_rows)

__all__ = ["BinaryPreferenceDataset", "PreferenceDataset", "HelpSteer3PreferenceDataset", "Tulu3PreferenceDataset",
           "PREFERENCE_DATASET_REGISTRY", "load_preference_dataset", "PreferenceSamples"]


def _pair(context, chosen: str, rejected: str, task: str) -> dict:
    return {"context": context,
            "completions": [{"rank": 0, "completion": [{"role": "assistant", "content": chosen}]},
                            {"rank": 1, "completion": [{"role": "assistant", "content": rejected}]}],
            "task_name": task}


def _as_turns(ctx):
    return list(ctx) if isinstance(ctx, list) else [{"role": "user", "content": ctx}]


class _PreferenceBase(RawDataset):
    def set_processor(self) -> None:
        self.processor = preference_preprocessor


class BinaryPreferenceDataset(_PreferenceBase):
    """``{prompt_key, chosen_key, rejected_key}`` rows (the prompt a string or a
    list of turns) from a local file or a hub id."""

    def __init__(self, data_path: str, prompt_key: str = "prompt", chosen_key: str = "chosen",
                 rejected_key: str = "rejected", subset: Optional[str] = None, split: Optional[str] = None,
                 split_validation_size: float = 0, seed: int = 42, **_):
        self.task_name = _task_name_of_path(data_path)
        keys = (prompt_key, chosen_key, rejected_key)
        task = self.task_name
        self.dataset = load_rows(data_path, subset, split).map(
            lambda r: _pair(_as_turns(r[keys[0]]), r[keys[1]], r[keys[2]], task))
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)


class PreferenceDataset(_PreferenceBase):
    """Rows already in the ``context`` / ``completions`` form."""

    def __init__(self, data_path: str, subset: Optional[str] = None, split: Optional[str] = None,
                 split_validation_size: float = 0, seed: int = 42, **_):
        self.task_name = _task_name_of_path(data_path)
        task = self.task_name
        self.dataset = load_rows(data_path, subset, split).map(lambda r: {**r, "task_name": task})
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)


class HelpSteer3PreferenceDataset(_HubResponseDataset, _PreferenceBase):
    """``nvidia/HelpSteer3`` preference subset: ``overall_preference`` < 0 prefers
    response1, > 0 response2; 0 (no preference) gives response1 as both sides,
    with a warning, as the reference does."""

    HUB = "nvidia/HelpSteer3"

    def __init__(self, split: str = "train", data_path: Optional[str] = None, **_):
        self.task_name = "HelpSteer3"
        self.dataset = self._load(data_path, "preference", split).map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        pref, r1, r2 = row["overall_preference"], row["response1"], row["response2"]
        if pref == 0:
            warnings.warn("HelpSteer3 row with overall_preference 0: response1 used as chosen and rejected",
                          stacklevel=2)
        chosen, rejected = (r2, r1) if pref > 0 else (r1, r1 if pref == 0 else r2)
        return _pair(_as_turns(row["context"]), chosen, rejected, self.task_name)

    set_processor = _PreferenceBase.set_processor


class Tulu3PreferenceDataset(_HubResponseDataset, _PreferenceBase):
    """``allenai/llama-3.1-tulu-3-8b-preference-mixture``: chosen / rejected
    conversations sharing every turn but the last (checked), whose last turns are
    the assistant's."""

    HUB = "allenai/llama-3.1-tulu-3-8b-preference-mixture"

    def __init__(self, split: str = "train", data_path: Optional[str] = None, **_):
        self.task_name = "Tulu3Preference"
        self.dataset = self._load(data_path, None, split).map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        ch, rj = row["chosen"], row["rejected"]
        if json.dumps(ch[:-1], ensure_ascii=False) != json.dumps(rj[:-1], ensure_ascii=False):
            raise ValueError(f"Tulu3 preference row: the chosen and rejected contexts differ ({ch} vs {rj})")
        if ch[-1]["role"] != "assistant" or rj[-1]["role"] != "assistant":
            raise ValueError("Tulu3 preference row: the last turns must be the assistant's")
        return _pair(list(ch[:-1]), ch[-1]["content"], rj[-1]["content"], self.task_name)

    set_processor = _PreferenceBase.set_processor


PREFERENCE_DATASET_REGISTRY: dict[str, Callable[..., RawDataset]] = {
    "HelpSteer3": HelpSteer3PreferenceDataset,
    "Tulu3Preference": Tulu3PreferenceDataset,
    "BinaryPreferenceDataset": BinaryPreferenceDataset,
    "PreferenceDataset": PreferenceDataset,
}


def load_preference_dataset(data_config: dict) -> RawDataset:
    """The preference dataset ``data_config["dataset_name"]`` names (a registry key
    or a dotted class path), with its task spec and ``preference_preprocessor``."""
    name = data_config["dataset_name"]
    if name in PREFERENCE_DATASET_REGISTRY:
        factory = PREFERENCE_DATASET_REGISTRY[name]
    elif "." in name:
        factory = _external_class(name)
    else:
        raise ValueError(f"unknown preference dataset {name!r}: use one of {sorted(PREFERENCE_DATASET_REGISTRY)} "
                         f"or a dotted path to a dataset class")
    ds = factory(**{k: v for k, v in data_config.items() if k != "dataset_name"})
    ds.set_task_spec(data_config)
    ds.set_processor()
    return ds


class PreferenceSamples:
    """A preference dataset as the DPO / RM loops' samples: each row through the
    dataset's processor (chat template, over-length masking), then split into the
    shared prompt tokens (the turns both logs have in common) and the chosen /
    rejected completion tokens."""

    def __init__(self, ds: RawDataset, tokenizer, max_seq_length: Optional[int] = None, split: str = "train"):
        self.rows = ds.dataset if split == "train" else ds.val_dataset
        self.ds, self.tokenizer, self.max_seq_length = ds, tokenizer, max_seq_length

    def __len__(self) -> int:
        return len(self.rows)

    def __getitem__(self, i: int) -> dict:
        import torch

        d = self.ds.processor(self.rows[i], self.ds.task_spec, self.tokenizer, self.max_seq_length, i)
        lc, lr = d["message_log_chosen"], d["message_log_rejected"]
        n = 0
        while n < min(len(lc), len(lr)) - 1 and torch.equal(lc[n]["token_ids"], lr[n]["token_ids"]):
            n += 1
        cat = lambda log: torch.cat([m["token_ids"] for m in log]) if log else torch.zeros(0, dtype=torch.long)
        return {"prompt": cat(lc[:n]), "chosen": cat(lc[n:]), "rejected": cat(lr[n:]), "idx": i,
                "loss_multiplier": d["loss_multiplier"]}
