"""Task specs and per-task data processors: raw dataset rows -> ``DatumSpec``.

Reference: ``nemo_rl/data/interfaces.py`` (``TaskDataSpec``, ``DatumSpec``) and
``nemo_rl/data/processors.py`` (``math_hf_data_processor`` ``:553`` is the
``default`` processor, ``math_data_processor`` ``:495``, ``sft_processor``
``:145``, ``preference_preprocessor`` ``:195``, ``multichoice_qa_processor``
``:855``, ``PROCESSOR_REGISTRY`` ``:1128``).  The registry names, the processor
call signature ``(datum_dict, task_data_spec, tokenizer, max_seq_length, idx)``
and the produced fields are kept, so custom processors written for the reference
plug in unchanged.

Shared rules (as the reference applies them):

* prompts render through the tokenizer's chat template with a generation prompt
  and are tokenised without extra special tokens;
* ``task_data_spec.prompt`` (from ``prompt_file``) is a ``str.format`` template
  with the problem as its argument; ``system_prompt`` becomes a system turn;
* a datum whose token count reaches ``max_seq_length`` is kept but masked:
  every message is cut to ``min(4, max_seq_length // n_messages)`` tokens and
  ``loss_multiplier`` is 0.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch

__all__ = ["TaskDataSpec", "PROCESSOR_REGISTRY", "register_processor", "math_hf_data_processor",
           "math_data_processor", "sft_processor", "multichoice_qa_processor", "preference_preprocessor",
           "helpsteer3_data_processor", "kd_data_processor", "nemo_gym_data_processor",
           "format_message_log"]


def _read(path: Optional[str]) -> Optional[str]:
    if path is None:
        return None
    if not os.path.exists(path):
        raise FileNotFoundError(f"prompt file {path} not found")
    with open(path, encoding="utf-8") as f:
        return f.read()


@dataclass
class TaskDataSpec:
    """Per-task prompt configuration; ``prompt`` / ``system_prompt`` are read from
    the files at construction."""

    task_name: Optional[str] = None
    prompt_file: Optional[str] = None
    system_prompt_file: Optional[str] = None
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        self.prompt = _read(self.prompt_file)
        self.system_prompt = _read(self.system_prompt_file)

    def copy_defaults(self, other: "TaskDataSpec") -> None:
        """Take ``other``'s prompt / system prompt where this spec has none."""
        if self.prompt is None:
            self.prompt = other.prompt
        if self.system_prompt is None:
            self.system_prompt = other.system_prompt


def _ids(tokenizer, text: str) -> torch.Tensor:
    out = tokenizer(text, return_tensors="pt", add_special_tokens=False)["input_ids"]
    return out[0] if isinstance(out, torch.Tensor) else torch.as_tensor(out[0], dtype=torch.int64)


def _prompt_messages(spec: TaskDataSpec, user_content: str) -> list[dict]:
    msgs = []
    if spec.system_prompt:
        msgs.append({"role": "system", "content": spec.system_prompt})
    msgs.append({"role": "user", "content": spec.prompt.format(user_content) if spec.prompt else user_content})
    return msgs


def _single_prompt_log(tokenizer, messages: list[dict]) -> list[dict]:
    text = tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                         add_special_tokens=False)
    return [{"role": "user", "content": text, "token_ids": _ids(tokenizer, text)}]


def _mask_if_long(message_log: list[dict], max_seq_length: Optional[int]) -> tuple[int, float]:
    length = sum(int(len(m["token_ids"])) for m in message_log)
    if max_seq_length is not None and length >= max_seq_length:
        keep = min(4, max_seq_length // max(1, len(message_log)))
        for m in message_log:
            m["token_ids"] = m["token_ids"][:keep]
        return length, 0.0
    return length, 1.0


def _datum(message_log, length, extra_env_info, loss_multiplier, idx, task_name=None) -> dict:
    d = {"message_log": message_log, "length": length, "extra_env_info": extra_env_info,
         "loss_multiplier": loss_multiplier, "idx": idx}
    if task_name is not None:
        d["task_name"] = task_name
    return d


def math_hf_data_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """Rows ``{"messages": [user problem, assistant answer], "task_name"}`` (the
    formatted response datasets) -> a one-message prompt with the answer as the
    environment's ground truth."""
    msgs = datum_dict["messages"]
    log = _single_prompt_log(tokenizer, _prompt_messages(task_data_spec, msgs[0]["content"]))
    length, lm = _mask_if_long(log, max_seq_length)
    return _datum(log, length, {"ground_truth": msgs[1]["content"]}, lm, idx, datum_dict.get("task_name"))


def math_data_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """Rows ``{"problem", "expected_answer"}`` -> prompt + ground truth."""
    log = _single_prompt_log(tokenizer, _prompt_messages(task_data_spec, datum_dict["problem"]))
    length, lm = _mask_if_long(log, max_seq_length)
    return _datum(log, length, {"ground_truth": str(datum_dict["expected_answer"])}, lm, idx,
                  datum_dict.get("task_name"))


def _multichoice_text(prompt: str, question: str, options: dict) -> str:
    lines = [f"{k}) {v}" for k, v in options.items() if v is not None]
    return prompt + f"\n\nQuestion: {question}\nOptions:\n" + "\n".join(lines)


def multichoice_qa_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """Rows ``{"question", "options": {letter: text}, "answer"[, "subject"]}``; the
    prompt template (when set) is followed by the question and lettered options."""
    q = datum_dict["question"]
    if task_data_spec.prompt:
        q = _multichoice_text(task_data_spec.prompt, q, datum_dict["options"])
    msgs = ([{"role": "system", "content": task_data_spec.system_prompt}] if task_data_spec.system_prompt else [])
    msgs.append({"role": "user", "content": q})
    log = _single_prompt_log(tokenizer, msgs)
    info = {"ground_truth": str(datum_dict["answer"])}
    if "subject" in datum_dict:
        info["subject"] = datum_dict["subject"]
    length = sum(int(len(m["token_ids"])) for m in log)
    return _datum(log, length, info, 1.0, idx, datum_dict.get("task_name"))


def format_message_log(messages: list[dict], tokenizer, task_data_spec: Optional[TaskDataSpec] = None,
                       add_bos_token: bool = True, add_eos_token: bool = True,
                       add_generation_prompt: bool = False, tools: Optional[list] = None) -> list[dict]:
    """Tokenise a conversation turn by turn with the chat template: turn ``i`` owns
    the text that rendering ``messages[:i+1]`` adds to rendering ``messages[:i]``,
    so the turns' token ids concatenate to the whole rendered conversation and
    each id is attributed to the turn that produced it (the loss mask needs
    that).  The system prompt of ``task_data_spec`` is prepended when the
    conversation has none; BOS / EOS are added once if the template left them
    out."""
    msgs = list(messages)
    if task_data_spec is not None and task_data_spec.system_prompt and (not msgs or msgs[0]["role"] != "system"):
        msgs = [{"role": "system", "content": task_data_spec.system_prompt}] + msgs
    kw = {"tools": tools} if tools else {}
    prev = ""
    out = []
    for i, m in enumerate(msgs):
        last = i == len(msgs) - 1
        text = tokenizer.apply_chat_template(msgs[:i + 1], tokenize=False,
                                             add_generation_prompt=add_generation_prompt and last,
                                             add_special_tokens=False, **kw)
        delta = text[len(prev):] if text.startswith(prev) else text
        prev = text
        ids = _ids(tokenizer, delta)
        if i == 0 and add_bos_token and getattr(tokenizer, "bos_token_id", None) is not None:
            if len(ids) == 0 or int(ids[0]) != tokenizer.bos_token_id:
                ids = torch.cat([torch.tensor([tokenizer.bos_token_id]), ids])
                delta = (getattr(tokenizer, "bos_token", "") or "") + delta
        if last and add_eos_token and getattr(tokenizer, "eos_token_id", None) is not None:
            if len(ids) == 0 or int(ids[-1]) != tokenizer.eos_token_id:
                ids = torch.cat([ids, torch.tensor([tokenizer.eos_token_id])])
                delta = delta + (getattr(tokenizer, "eos_token", "") or "")
        out.append({"role": m["role"], "content": delta, "token_ids": ids.to(torch.int64)})
    return out


def sft_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int,
                  add_bos: bool = True, add_eos: bool = True, add_generation_prompt: bool = False):
    """Rows ``{"messages": [...]}[, "tools"]`` -> per-turn tokenised message log
    (the SFT loss trains on the assistant turns)."""
    log = format_message_log(datum_dict["messages"], tokenizer, task_data_spec, add_bos_token=add_bos,
                             add_eos_token=add_eos, add_generation_prompt=add_generation_prompt,
                             tools=datum_dict.get("tools"))
    length, lm = _mask_if_long(log, max_seq_length)
    return _datum(log, length, None, lm, idx, datum_dict.get("task_name"))


def preference_preprocessor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """Rows ``{"context": [...], "completions": [{"rank", "completion": [...]}] x 2}``
    (lower rank preferred) -> chosen / rejected message logs sharing the context.
    Pairs too long for ``max_seq_length`` are truncated and masked."""
    comps = datum_dict["completions"]
    if len(comps) != 2:
        raise ValueError("preference training takes exactly two completions per context")
    chosen, rejected = sorted(comps, key=lambda c: c["rank"])
    ctx = datum_dict["context"]
    log_c = format_message_log(ctx + chosen["completion"], tokenizer, task_data_spec)
    log_r = format_message_log(ctx + rejected["completion"], tokenizer, task_data_spec)
    len_c = sum(int(len(m["token_ids"])) for m in log_c)
    len_r = sum(int(len(m["token_ids"])) for m in log_r)
    lm = 1.0
    if max_seq_length is not None and max(len_c, len_r) > max_seq_length:
        for log in (log_c, log_r):
            keep = min(4, max_seq_length // max(1, len(log)))
            for m in log:
                m["token_ids"] = m["token_ids"][:keep]
        lm = 0.0
    out = {"message_log_chosen": log_c, "message_log_rejected": log_r, "length_chosen": len_c,
           "length_rejected": len_r, "loss_multiplier": lm, "idx": idx}
    if "task_name" in datum_dict:
        out["task_name"] = datum_dict["task_name"]
    return out


def helpsteer3_data_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """HelpSteer3 rows for RL with a reward-model environment: ``context`` (a
    string or a list of turns) is the prompt; the preferred response is kept as
    ``extra_env_info["ground_truth"]``."""
    ctx = datum_dict.get("context") or datum_dict.get("messages")
    msgs = [{"role": "user", "content": ctx}] if isinstance(ctx, str) else list(ctx)
    if task_data_spec.system_prompt and msgs[0]["role"] != "system":
        msgs = [{"role": "system", "content": task_data_spec.system_prompt}] + msgs
    log = _single_prompt_log(tokenizer, msgs)
    length, lm = _mask_if_long(log, max_seq_length)
    gt = datum_dict.get("response") or datum_dict.get("ground_truth")
    return _datum(log, length, {"ground_truth": gt}, lm, idx, datum_dict.get("task_name"))


def kd_data_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """Distillation prompts: the user turn of ``messages`` (or ``problem``) as the
    prompt; no ground truth needed (the teacher supplies the targets)."""
    if "messages" in datum_dict:
        msgs = datum_dict["messages"]
        # raw-text rows (one assistant turn, e.g. ``arrow_text``) use the text itself
        user = next((m["content"] for m in msgs if m["role"] == "user"), msgs[0]["content"] if msgs else "")
    else:
        user = datum_dict["problem"]
    log = _single_prompt_log(tokenizer, _prompt_messages(task_data_spec, user))
    length, lm = _mask_if_long(log, max_seq_length)
    return _datum(log, length, {}, lm, idx, datum_dict.get("task_name"))


def nemo_gym_data_processor(datum_dict: dict, task_data_spec: TaskDataSpec, tokenizer, max_seq_length, idx: int):
    """NeMo-Gym rows: the Gym server builds the prompt, so the datum carries the
    parsed ``extra_env_info`` payload and one empty user turn (length 0).

    Reference: ``nemo_rl/data/processors.py:932`` (text rows; the video and image
    tiling branches belong to the multimodal path)."""
    import json

    import torch

    info = datum_dict["extra_env_info"]
    if isinstance(info, (str, bytes)):
        info = json.loads(info)
    log = [{"role": "user", "content": "", "token_ids": torch.empty(0, dtype=torch.long)}]
    return _datum(log, 0, info, 1.0, idx, datum_dict.get("task_name"))


PROCESSOR_REGISTRY: dict[str, Callable[..., dict]] = {
    "default": math_hf_data_processor,
    "math_hf_data_processor": math_hf_data_processor,
    "math_data_processor": math_data_processor,
    "sft_processor": sft_processor,
    "multichoice_qa_processor": multichoice_qa_processor,
    "helpsteer3_data_processor": helpsteer3_data_processor,
    "kd_data_processor": kd_data_processor,
    "chat_kd_processor": kd_data_processor,
    "nemo_gym_data_processor": nemo_gym_data_processor,
}


def register_processor(name: str, fn: Callable[..., dict]) -> None:
    """Add a processor under ``name`` (names are unique)."""
    if name in PROCESSOR_REGISTRY:
        raise ValueError(f"processor {name!r} is already registered")
    PROCESSOR_REGISTRY[name] = fn


def get_processor(name: str) -> Callable[..., Any]:
    if name not in PROCESSOR_REGISTRY:
        raise KeyError(f"processor {name!r} not registered; known: {sorted(PROCESSOR_REGISTRY)} "
                       f"(register_processor adds one)")
    return PROCESSOR_REGISTRY[name]
