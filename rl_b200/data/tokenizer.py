"""Tokenizers and chat templates for the data pipeline.

``get_tokenizer(tokenizer_config)`` follows the reference's contract
(``nemo_rl/algorithms/utils.py:357``): ``name`` is a tokenizer path (a local
Hugging Face model / tokenizer directory; this image has no network, so hub
names resolve only from a local cache), ``chat_template`` selects the template:

* key absent or ``"default"`` - the tokenizer's own template;
* ``None`` - passthrough: the concatenated message contents;
* any other string - a custom Jinja template (or the name of one of
  ``COMMON_CHAT_TEMPLATES``);

and a missing pad token becomes the EOS token.

``ByteTokenizer`` is a self-contained byte-level tokenizer with the same call
surface the data pipeline uses (``apply_chat_template``, ``__call__``,
``encode`` / ``decode``, ``eos_token_id`` / ``pad_token_id``).  It needs no
files, so the tiny CPU configs and tests run the real text pipeline (chat
rendering, tokenisation, math verification of decoded answers) offline.
``name: byte`` selects it.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

__all__ = ["COMMON_CHAT_TEMPLATES", "ByteTokenizer", "get_tokenizer", "render_chat"]

# Named templates usable as ``tokenizer.chat_template: <name>``.
COMMON_CHAT_TEMPLATES = {
    # contents only, no role markers (what ``chat_template: null`` selects)
    "passthrough": "{% for message in messages %}{{ message['content'] }}{% endfor %}",
    # plain role-tagged turns; a trailing assistant header when a generation prompt is asked for
    "simple_role": (
        "{% for message in messages %}{{ '<|' + message['role'] + '|>\n' + message['content'] + '\n' }}{% endfor %}"
        "{% if add_generation_prompt %}{{ '<|assistant|>\n' }}{% endif %}"
    ),
}


def render_chat(template: str, messages: list[dict], add_generation_prompt: bool = False, **extra) -> str:
    """Render ``messages`` with a Jinja chat template (sandboxed environment, as
    Hugging Face tokenizers do)."""
    from jinja2.sandbox import ImmutableSandboxedEnvironment

    env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
    return env.from_string(template).render(messages=messages, add_generation_prompt=add_generation_prompt, **extra)


class ByteTokenizer:
    """UTF-8 bytes as tokens: id = byte + 3; 0 = pad, 1 = bos, 2 = eos.
    ``vocab_size`` is 259, so any model with at least that many embedding rows
    can read it."""

    pad_token_id = 0
    bos_token_id = 1
    eos_token_id = 2
    pad_token = "<pad>"
    bos_token = "<s>"
    eos_token = "</s>"
    vocab_size = 259
    name_or_path = "byte"

    def __init__(self, chat_template: Optional[str] = None):
        self.chat_template = chat_template if chat_template is not None else COMMON_CHAT_TEMPLATES["simple_role"]

    def __len__(self) -> int:
        return self.vocab_size

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids = [b + 3 for b in text.encode("utf-8")]
        return ([self.bos_token_id] + ids) if add_special_tokens else ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        if isinstance(ids, torch.Tensor):
            ids = ids.tolist()
        out = bytearray()
        for i in ids:
            i = int(i)
            if i >= 3 and i < 259:
                out.append(i - 3)
            elif not skip_special_tokens:
                out.extend({0: b"<pad>", 1: b"<s>", 2: b"</s>"}.get(i, b""))
        return out.decode("utf-8", errors="replace")

    def batch_decode(self, seqs, skip_special_tokens: bool = True) -> list[str]:
        return [self.decode(s, skip_special_tokens) for s in seqs]

    def __call__(self, text, return_tensors: Optional[str] = None, add_special_tokens: bool = False, **_):
        if isinstance(text, str):
            ids = self.encode(text, add_special_tokens)
            return {"input_ids": torch.tensor([ids], dtype=torch.int64) if return_tensors == "pt" else ids}
        seqs = [self.encode(t, add_special_tokens) for t in text]
        return {"input_ids": seqs}

    def apply_chat_template(self, messages: list[dict], tokenize: bool = True, add_generation_prompt: bool = False,
                            add_special_tokens: bool = False, **kw):
        text = render_chat(self.chat_template, messages, add_generation_prompt=add_generation_prompt,
                           bos_token=self.bos_token, eos_token=self.eos_token, **kw)
        return self.encode(text) if tokenize else text


def _resolve_template(t: str) -> str:
    return COMMON_CHAT_TEMPLATES.get(t, t)


def get_tokenizer(tokenizer_config: dict | str, get_processor: bool = False) -> Any:
    """Tokenizer for ``tokenizer_config`` (see the module docstring)."""
    if isinstance(tokenizer_config, str):
        tokenizer_config = {"name": tokenizer_config}
    name = tokenizer_config["name"]
    has_key = "chat_template" in tokenizer_config
    tmpl = tokenizer_config.get("chat_template", "default")
    if name == "byte":
        if has_key and tmpl is None:
            return ByteTokenizer(COMMON_CHAT_TEMPLATES["passthrough"])
        return ByteTokenizer(None if tmpl in (None, "default") else _resolve_template(tmpl))
    kwargs = dict(tokenizer_config.get("tokenizer_kwargs") or {})
    if get_processor:
        from transformers import AutoProcessor

        proc = AutoProcessor.from_pretrained(name, trust_remote_code=True, **kwargs)
        tok = proc.tokenizer
    else:
        from transformers import AutoTokenizer

        tok = proc = AutoTokenizer.from_pretrained(name, trust_remote_code=True, **kwargs)
    if tok.pad_token is None:
        tok.pad_token = tok.eos_token
    if has_key and tmpl is None:
        tok.chat_template = COMMON_CHAT_TEMPLATES["passthrough"]
    elif tmpl not in (None, "default"):
        tok.chat_template = _resolve_template(tmpl)
    return proc
