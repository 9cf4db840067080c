"""Checkpoint tokenization without executing tokenizer code from the checkpoint.

Same public API as ``dsv41_train/rl/tokenizer.py`` (``ModelTokenizer.encode_prompt``,
``encode_conversation``, ``encode_completion``, ``decode``, ``eos_token_ids``,
``read_eos_token_ids``): ``tokenizer.json`` through the ``tokenizers`` library and the
checkpoint's chat template rendered by a sandboxed jinja2 environment, then tokenized without
added special tokens (what HF ``apply_chat_template`` does).
"""

from __future__ import annotations

import json
from pathlib import Path

from jinja2 import TemplateError
from jinja2.sandbox import ImmutableSandboxedEnvironment
from tokenizers import Tokenizer


def _read_json(directory: Path, name: str) -> dict:
    path = directory / name
    if not path.exists():
        return {}
    try:
        value = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, ValueError) as error:
        raise ValueError(f"cannot read {path}: {error}") from error
    if not isinstance(value, dict):
        raise ValueError(f"{path} must contain a JSON object")
    return value


def _token_ids(value, name: str) -> tuple[int, ...]:
    values = value if isinstance(value, (list, tuple)) else [value]
    if not values or any(type(v) is not int or v < 0 for v in values):
        raise ValueError(f"{name} must be a nonnegative integer or a nonempty list of them")
    return tuple(dict.fromkeys(values))


def read_eos_token_ids(model_dir, fallback=None) -> tuple[int, ...]:
    """Stop ids from generation_config.json, config.json or its text_config (first present)."""
    directory = Path(model_dir)
    config = _read_json(directory, "config.json")
    text = config.get("text_config", {}) if isinstance(config.get("text_config", {}), dict) else {}
    for source in (_read_json(directory, "generation_config.json"), config, text):
        if source.get("eos_token_id") is not None:
            return _token_ids(source["eos_token_id"], "eos_token_id")
    return () if fallback is None else _token_ids(fallback, "eos_token_id")


def _chat_template(directory: Path, config: dict) -> str | None:
    path = directory / "chat_template.jinja"
    template = path.read_text(encoding="utf-8") if path.exists() else config.get("chat_template")
    if template is None:
        return None
    if isinstance(template, list):
        choices = {}
        for entry in template:
            if not isinstance(entry, dict) or not isinstance(entry.get("name"), str) or entry["name"] in choices:
                raise ValueError("chat template list must contain unique named templates")
            choices[entry["name"]] = entry["template"]
        template = choices
    if isinstance(template, dict):
        if "default" not in template:
            raise ValueError("named chat templates require a 'default' template")
        template = template["default"]
    if not isinstance(template, str) or not template.strip():
        raise ValueError("chat template must be a nonempty string")
    return template


def _token_text(value):
    if isinstance(value, dict):
        return value.get("content")
    return value


class ModelTokenizer:
    def __init__(self, model_dir):
        directory = Path(model_dir)
        path = directory / "tokenizer.json"
        if not path.is_file():
            raise ValueError(f"{path} is required; only local tokenizers tokenizer.json checkpoints are supported")
        try:
            self._tokenizer = Tokenizer.from_file(str(path))
        except Exception as error:
            raise ValueError(f"unsupported or invalid tokenizer.json at {path}: {error}") from error
        vocabulary = self._tokenizer.get_vocab(with_added_tokens=True)
        self._vocabulary_ids = set(vocabulary.values())
        config = _read_json(directory, "config.json")
        text_config = config.get("text_config", {}) if isinstance(config.get("text_config", {}), dict) else {}
        tok_config = _read_json(directory, "tokenizer_config.json")
        self._template_source = _chat_template(directory, tok_config)
        vocab_size = config.get("vocab_size", text_config.get("vocab_size"))
        if vocab_size is not None and any(i >= vocab_size for i in vocabulary.values()):
            raise ValueError("tokenizer vocabulary contains IDs outside the model vocabulary")
        self.special = {}
        for name in ("bos_token", "eos_token", "pad_token", "unk_token"):
            text = _token_text(tok_config.get(name))
            if text is None:
                value = tok_config.get(name + "_id", config.get(name + "_id", text_config.get(name + "_id")))
                if value is not None:
                    text = self._tokenizer.id_to_token(_token_ids(value, name)[0])
            self.special[name] = text
        fallback = None
        if self.special["eos_token"] is not None:
            fallback = self._tokenizer.token_to_id(self.special["eos_token"])
        self._eos_token_ids = read_eos_token_ids(directory, fallback=fallback)
        for token_id in self._eos_token_ids:
            self._validate_id(token_id, "eos_token_id")
        self.add_bos = bool(tok_config.get("add_bos_token", False))
        self._env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)

        def raise_exception(message):
            raise TemplateError(message)

        self._env.globals["raise_exception"] = raise_exception
        self._template = self._env.from_string(self._template_source) if self._template_source else None

    @property
    def eos_token_ids(self) -> tuple[int, ...]:
        return self._eos_token_ids

    @property
    def pad_token_id(self) -> int | None:
        text = self.special.get("pad_token")
        return None if text is None else self._tokenizer.token_to_id(text)

    def _validate_id(self, token_id, name):
        if type(token_id) is not int or token_id not in self._vocabulary_ids:
            raise ValueError(f"{name} contains an ID outside the tokenizer vocabulary: {token_id!r}")

    def encode_text(self, text: str, *, add_special_tokens: bool = False) -> list[int]:
        return self._tokenizer.encode(text, add_special_tokens=add_special_tokens).ids

    def encode_prompt(self, prompt: str | None = None, messages: list[dict] | None = None) -> list[int]:
        if (prompt is None) == (messages is None):
            raise ValueError("provide exactly one of prompt or messages")
        if prompt is not None:
            if not isinstance(prompt, str) or not prompt.strip():
                raise ValueError("prompt must be a nonempty string")
            if self._template is None:
                return self.encode_text(prompt, add_special_tokens=True)
            messages = [{"role": "user", "content": prompt}]
        if self._template is None:
            raise ValueError("messages require a checkpoint chat template")
        self._check_messages(messages, final_user=True)
        return self._encode_template(messages)

    def encode_conversation(self, messages, *, tools=None, chat_template_kwargs=None) -> list[int]:
        if self._template is None:
            raise ValueError("conversations require a checkpoint chat template")
        options = dict(chat_template_kwargs or {})
        if set(options) - {"enable_thinking"}:
            raise ValueError("chat_template_kwargs support only enable_thinking")
        if not isinstance(messages, list) or not messages:
            raise ValueError("messages must be a nonempty list")
        if messages[-1].get("role") not in ("user", "tool"):
            raise ValueError("conversations must end with a user message or completed tool results")
        return self._encode_template(messages, tools=tools, **options)

    def encode_completion(self, messages, answer: str, *, chat_template_kwargs=None) -> tuple[list[int], list[int]]:
        """(generation prompt ids, completed conversation ids); the prompt must be a token prefix."""
        if not isinstance(answer, str) or not answer.strip():
            raise ValueError("answer must be a nonempty string")
        prompt_ids = self.encode_conversation(messages, chat_template_kwargs=chat_template_kwargs)
        full_ids = self._encode_template([*messages, {"role": "assistant", "content": answer}],
                                         add_generation_prompt=False, **(chat_template_kwargs or {}))
        if full_ids[:len(prompt_ids)] != prompt_ids:
            raise ValueError("completed conversation does not preserve the generation prompt token prefix")
        return prompt_ids, full_ids

    def _check_messages(self, messages, *, final_user: bool):
        if not isinstance(messages, list) or not messages:
            raise ValueError("messages must be a nonempty list")
        for m in messages:
            if not isinstance(m, dict) or set(m) != {"role", "content"}:
                raise ValueError("messages support only role and content")
            if m["role"] not in ("system", "user", "assistant"):
                raise ValueError("message role must be system, user, or assistant")
            if not isinstance(m["content"], str) or not m["content"].strip():
                raise ValueError("message content must be nonempty text")
        if final_user and messages[-1]["role"] != "user":
            raise ValueError("messages must end with a user message for generation")

    def _encode_template(self, messages, *, add_generation_prompt=True, tools=None, **kwargs):
        try:
            text = self._template.render(messages=messages, add_generation_prompt=add_generation_prompt,
                                         tools=tools, **{k: v for k, v in self.special.items() if v is not None},
                                         **kwargs)
        except (TemplateError, TypeError, ValueError) as error:
            raise ValueError(f"cannot render checkpoint chat template: {error}") from error
        ids = self.encode_text(text)
        if not ids:
            raise ValueError("chat template must produce a nonempty list of token IDs")
        return ids

    def decode(self, ids, *, skip_special_tokens=True) -> str:
        ids = list(ids)
        for i in ids:
            self._validate_id(i, "decoded token IDs")
        return self._tokenizer.decode(ids, skip_special_tokens=skip_special_tokens)


__all__ = ["ModelTokenizer", "read_eos_token_ids"]
