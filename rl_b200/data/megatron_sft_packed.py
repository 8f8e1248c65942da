"""Megatron-LM offline-packed SFT rows (``.jsonl.packed``).

Reference: ``nemo_rl/data/megatron_sft_packed.py`` (``megatron_sft_packed_preprocessor``
``:298``, prompt formats ``:46``, per-turn label masking ``:187``) and the
dataset ``nemo_rl/data/datasets/response_datasets/megatron_sft_packed.py:29``.

A packed record is a list of messages in which every ``system`` message starts a
new conversation.  Each conversation is rendered in one of the prompt formats
below and tokenised; prompt tokens (system / user / tool turns, and the first
``assistant_prefix_len`` tokens of an assistant turn) get the ignore label.  The
conversations are concatenated (each padded to a multiple of ``2 * cp`` under
context parallelism, positions restarting at 0 per conversation) into one row of
``max_seq_length + 1`` tokens, padded or cut at the end; the row is then
pre-shifted: ``input_ids = pack[:-1]``, ``target_ids = pack[1:]``, with
``token_mask`` 0 where the target is the ignore label or the pad token, and
``packed_cu_seqlens`` the conversation boundaries.

How this framework trains on such a row: attention never crosses a boundary, so
segment ``k`` (``pack[cu[k] : cu[k+1]]``) is an independent sequence, except that
its last position predicts ``pack[cu[k+1]]`` (the next segment's first token, as
the pre-shifted targets say).  The preprocessor therefore also emits
``packed_segments``: for each segment the tokens ``pack[cu[k] : cu[k+1] + 1]``
(one extra trailing token) and a mask whose entry ``j`` says whether the target
of input position ``j - 1`` counts.  The policy worker packs those sequences THD
with its own cu_seqlens, and the next-token log-prob at each (position, target)
pair is exactly the direct path's, so ``NLLLossFn`` gives the same loss.

Design difference: conversations are tokenised turn by turn (each rendered turn
encoded on its own and the pieces concatenated), which makes the label
boundaries exact by construction; the reference tokenises the whole rendering
and raises if its per-turn re-tokenisation disagrees.
"""

from __future__ import annotations

import warnings
from dataclasses import dataclass, replace
from typing import Any, Callable, Optional

import torch

__all__ = ["IGNORE_INDEX", "PROMPT_FORMATS", "PromptFormat", "resolve_prompt_format",
           "split_packed_conversations", "tokenize_conversation", "megatron_sft_packed_preprocessor",
           "cp_granularity"]

IGNORE_INDEX = -100


def _strip_think(s: str) -> str:
    return s.replace("/think", "").replace("/no_think", "").strip()


def _render_identity(role: str, content: str) -> str:
    return content


def _render_nano_v2(role: str, content: str) -> str:
    if role == "system":
        return "<SPECIAL_10>System\n" + _strip_think(content) + "\n"
    if role == "user":
        return "<SPECIAL_11>User\n" + _strip_think(content) + "\n"
    if role == "assistant":
        return "<SPECIAL_11>Assistant\n" + content.strip() + "\n<SPECIAL_12>\n"
    return ""


def _render_h_aligned(role: str, content: str) -> str:
    if role == "system":
        return "<SPECIAL_10>System\n" + content.strip() + "\n"
    if role == "user":
        return "<SPECIAL_11>User\n" + content.strip() + "\n<SPECIAL_11>Assistant\n"
    if role == "assistant":
        return content.strip() + "\n"
    return ""


@dataclass(frozen=True)
class PromptFormat:
    """One prompt format: how a turn renders, how many leading tokens of an
    assistant turn are prompt (its header), and the pad token's name."""

    render: Callable[[str, str], str]
    assistant_prefix_len: int
    pad_token: Optional[str]
    has_system_role: bool = True


PROMPT_FORMATS = {
    "identity": PromptFormat(_render_identity, 0, "<unk>"),
    "nemotron-nano-v2": PromptFormat(_render_nano_v2, 3, "<unk>"),
    "nemotron-h-aligned": PromptFormat(_render_h_aligned, 0, "<SPECIAL_233>"),
}


def resolve_prompt_format(name: str, override_pad_token: Optional[str] = None) -> PromptFormat:
    if name not in PROMPT_FORMATS:
        raise NotImplementedError(f"unknown SFT prompt format {name!r}: one of {sorted(PROMPT_FORMATS)}")
    fmt = PROMPT_FORMATS[name]
    return fmt if override_pad_token is None else replace(fmt, pad_token=override_pad_token)


def cp_granularity(context_parallel_size: int) -> int:
    """Token multiple of every segment under context parallelism (each document
    is cut into ``2 * cp`` load-balanced chunks)."""
    return 2 * int(context_parallel_size)


def split_packed_conversations(messages: list[dict]) -> list[list[dict]]:
    """Cut a packed message list before every ``system`` message."""
    convs: list[list[dict]] = []
    for m in messages:
        if m["role"] == "system" or not convs:
            convs.append([m])
        else:
            convs[-1].append(m)
    return convs


def _encode(tokenizer, text: str) -> list[int]:
    ids = tokenizer.encode(text, add_special_tokens=False)
    if isinstance(ids, torch.Tensor):
        ids = ids.tolist()
    return [int(i) for i in ids]


def tokenize_conversation(conv: list[dict], tokenizer, fmt_name: str,
                          fmt: Optional[PromptFormat] = None) -> tuple[list[int], list[int]]:
    """(tokens, labels) of one conversation: labels are the tokens with prompt
    positions set to ``IGNORE_INDEX`` (the ``identity`` format trains on every
    token)."""
    fmt = fmt or resolve_prompt_format(fmt_name)
    if not fmt.has_system_role and conv and conv[0]["role"] == "system":
        conv = conv[1:]
    tokens: list[int] = []
    labels: list[int] = []
    for i, turn in enumerate(conv):
        role = turn["role"].lower()
        if role not in ("system", "user", "tool", "assistant"):
            raise ValueError(f"unknown role {turn['role']!r} in a packed SFT conversation")
        if role == "assistant":
            if not turn["content"]:
                raise ValueError("empty assistant turn in a packed SFT conversation")
            if i == 0 or conv[i - 1]["role"].lower() not in ("user", "tool"):
                raise ValueError("an assistant turn must follow a user or tool turn")
        ids = _encode(tokenizer, fmt.render(role, turn["content"]))
        tokens += ids
        if fmt_name == "identity":
            labels += ids
        elif role == "assistant":
            if fmt.assistant_prefix_len > len(ids):
                raise ValueError(f"assistant_prefix_len={fmt.assistant_prefix_len} exceeds the turn's "
                                 f"{len(ids)} tokens")
            labels += [IGNORE_INDEX] * fmt.assistant_prefix_len + ids[fmt.assistant_prefix_len:]
        else:
            labels += [IGNORE_INDEX] * len(ids)
    return tokens, labels


def _pad_id(tokenizer, fmt: PromptFormat) -> int:
    pad = None
    if fmt.pad_token is not None and hasattr(tokenizer, "convert_tokens_to_ids"):
        pad = tokenizer.convert_tokens_to_ids(fmt.pad_token)
        unk = getattr(tokenizer, "unk_token_id", None)
        if pad is not None and unk is not None and pad == unk and fmt.pad_token != getattr(tokenizer, "unk_token", None):
            pad = None  # the name is not in this vocabulary
    if pad is None:
        pad = getattr(tokenizer, "pad_token_id", None)
    if pad is None:
        raise ValueError("packed SFT data needs a pad token distinct from EOS")
    eos = getattr(tokenizer, "eos_token_id", None)
    if eos is not None and int(pad) == int(eos):
        raise ValueError("packed SFT data needs a pad token distinct from EOS")
    return int(pad)


def megatron_sft_packed_preprocessor(datum_dict: dict, task_data_spec, tokenizer, max_seq_length: int, idx: int, *,
                                     prompt_format: str, context_parallel_size: int = 1,
                                     pad_token: Optional[str] = None, **_: Any) -> dict:
    """One packed record -> one pre-shifted row of ``max_seq_length`` positions
    plus its ``packed_segments`` (see the module docstring)."""
    if max_seq_length is None or int(max_seq_length) < 1:
        raise ValueError("max_seq_length must be a positive integer")
    L = int(max_seq_length)
    cp = int(context_parallel_size)
    if cp < 1:
        raise ValueError("context_parallel_size must be >= 1")
    gran = cp_granularity(cp)
    if cp > 1 and L % gran:
        raise ValueError(f"max_seq_length={L} must be a multiple of 2 * context_parallel_size ({gran})")
    fmt = resolve_prompt_format(prompt_format, pad_token)
    pad = _pad_id(tokenizer, fmt)
    convs = split_packed_conversations(datum_dict["packed_messages"])
    if not convs:
        raise ValueError("a packed SFT record needs at least one conversation")
    toks: list[int] = []
    labs: list[int] = []
    pos: list[int] = []
    cu = [0]

    def pad_to(n: int) -> None:  # padding continues the last conversation's positions
        start = pos[-1] + 1
        toks.extend([pad] * n)
        labs.extend([pad] * n)
        pos.extend(range(start, start + n))

    cut = False
    dropped = 0
    for ci, conv in enumerate(convs):
        t, lab = tokenize_conversation(conv, tokenizer, prompt_format, fmt)
        if not t:
            raise ValueError("a packed SFT conversation tokenised to zero tokens")
        toks += t
        labs += lab
        pos += range(len(t))
        if cp > 1 and len(toks) % gran:
            pad_to(gran - len(toks) % gran)
        cu.append(len(toks))
        if len(toks) == L:
            dropped = len(convs) - ci - 1
            break
        if len(toks) > L:  # cut to L tokens plus one pad (the last target)
            toks, labs, pos = toks[:L] + [pad], labs[:L] + [pad], pos[:L + 1]
            cu[-1] = L
            cut, dropped = True, len(convs) - ci - 1
            break
    if cut or dropped:
        warnings.warn(f"packed SFT row {idx} overflowed max_seq_length={L}: "
                      f"{'the last conversation was cut and ' if cut else ''}{dropped} of {len(convs)} "
                      f"conversations dropped (the tokenizer / pack length differ from the offline packer's)",
                      stacklevel=2)
    if len(toks) < L + 1:
        pad_to(L + 1 - len(toks))
        cu[-1] = len(toks) - 1
    assert len(toks) == len(labs) == len(pos) == L + 1
    input_ids = torch.tensor(toks[:-1], dtype=torch.int64)
    target_ids = torch.tensor(labs[1:], dtype=torch.int64)
    token_mask = ((target_ids != pad) & (target_ids != IGNORE_INDEX)).float()
    cu_t = torch.tensor(cu, dtype=torch.int32)
    seg = cu_t[1:] - cu_t[:-1]
    if cp > 1 and bool((seg % gran != 0).any()):
        raise ValueError(f"packed segment lengths must be multiples of {gran} under context_parallel_size={cp}")
    # the same row as independent sequences: segment k's tokens plus the next token,
    # mask[j] = token_mask[cu[k] + j - 1] (whether input position j - 1's target counts)
    full = torch.tensor(toks, dtype=torch.int64)
    segments = []
    for k in range(len(cu) - 1):
        a, b = cu[k], cu[k + 1]
        m = torch.zeros(b - a + 1, dtype=torch.float32)
        m[1:] = token_mask[a:b]
        segments.append({"token_ids": full[a:b + 1].clone(), "token_loss_mask": m})
    return {
        "message_log": [], "length": L, "extra_env_info": None, "loss_multiplier": 1.0, "idx": idx,
        "task_name": datum_dict.get("task_name", "megatron_sft_packed"),
        "input_ids": input_ids, "target_ids": target_ids, "token_mask": token_mask,
        "position_ids": torch.tensor(pos[:-1], dtype=torch.int64), "packed_cu_seqlens": cu_t,
        "packed_max_seqlen": int(seg.max()), "packed_context_parallel_size": cp,
        "packed_segments": segments,
    }
