"""Tokenization of a checkpoint directory without running any code the checkpoint ships.

Public API of ``dsv41_train/rl/tokenizer.py`` (``ModelTokenizer.encode_prompt``,
``encode_conversation``, ``encode_completion``, ``decode``, ``eos_token_ids``,
``read_eos_token_ids``). ``tokenizer.json`` is read by the ``tokenizers`` library; the chat
template (``chat_template.jinja``, or ``chat_template`` in tokenizer_config.json, possibly a list
of named templates with a ``default``) is rendered in a sandboxed, immutable jinja2 environment
and the rendered text is tokenized without added special tokens - what HF
``apply_chat_template`` does.
"""

from __future__ import annotations

import json
from pathlib import Path

from jinja2 import TemplateError
from jinja2.sandbox import ImmutableSandboxedEnvironment
from tokenizers import Tokenizer

_SPECIAL = ("bos_token", "eos_token", "pad_token", "unk_token")
_ROLES = ("system", "user", "assistant")


def _json_object(directory: Path, name: str) -> dict:
    """The JSON object in ``directory/name``, or {} when the file does not exist."""
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


def _nested(config: dict) -> dict:
    text = config.get("text_config", {})
    return text if isinstance(text, dict) else {}


def _id_tuple(value, name: str) -> tuple[int, ...]:
    items = list(value) if isinstance(value, (list, tuple)) else [value]
    if not items or not all(type(i) is int and i >= 0 for i in items):
        raise ValueError(f"{name} must be a nonnegative integer or a nonempty list of them")
    return tuple(dict.fromkeys(items))  # distinct, first occurrence order


def read_eos_token_ids(model_dir, fallback=None) -> tuple[int, ...]:
    """Stop ids from the first of generation_config.json, config.json and its text_config that
    names them; else ``fallback`` (or none)."""
    directory = Path(model_dir)
    config = _json_object(directory, "config.json")
    for source in (_json_object(directory, "generation_config.json"), config, _nested(config)):
        if source.get("eos_token_id") is not None:
            return _id_tuple(source["eos_token_id"], "eos_token_id")
    return () if fallback is None else _id_tuple(fallback, "eos_token_id")


def _template_source(directory: Path, tokenizer_config: dict) -> str | None:
    file = directory / "chat_template.jinja"
    template = file.read_text(encoding="utf-8") if file.exists() else tokenizer_config.get("chat_template")
    if template is None:
        return None
    if isinstance(template, list):  # named templates
        named = {}
        for entry in template:
            name = entry.get("name") if isinstance(entry, dict) else None
            if not isinstance(name, str) or name in named:
                raise ValueError("chat template list must contain unique named templates")
            named[name] = entry["template"]
        template = named
    if isinstance(template, dict):
        if "default" not in template:
            raise ValueError("named chat templates require a 'default' template")
        template = template["default"]
    if not (isinstance(template, str) and template.strip()):
        raise ValueError("chat template must be a nonempty string")
    return template


def _raise_from_template(message):
    raise TemplateError(message)


class ModelTokenizer:
    def __init__(self, model_dir):
        directory = Path(model_dir)
        vocab_file = directory / "tokenizer.json"
        if not vocab_file.is_file():
            raise ValueError(f"{vocab_file} is required; only local tokenizers tokenizer.json checkpoints are supported")
        try:
            self._tokenizer = Tokenizer.from_file(str(vocab_file))
        except Exception as error:
            raise ValueError(f"unsupported or invalid tokenizer.json at {vocab_file}: {error}") from error
        known = set(self._tokenizer.get_vocab(with_added_tokens=True).values())
        self._known_ids = known
        config = _json_object(directory, "config.json")
        tokenizer_config = _json_object(directory, "tokenizer_config.json")
        model_vocab = config.get("vocab_size", _nested(config).get("vocab_size"))
        if model_vocab is not None and max(known, default=-1) >= model_vocab:
            raise ValueError("tokenizer vocabulary contains IDs outside the model vocabulary")
        self.special = {name: self._special_text(name, tokenizer_config, config) for name in _SPECIAL}
        eos_text = self.special["eos_token"]
        fallback = None if eos_text is None else self._tokenizer.token_to_id(eos_text)
        self._eos_token_ids = read_eos_token_ids(directory, fallback=fallback)
        for token_id in self._eos_token_ids:
            self._check_id(token_id, "eos_token_id")
        self.add_bos = bool(tokenizer_config.get("add_bos_token", False))
        source = _template_source(directory, tokenizer_config)
        environment = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
        environment.globals["raise_exception"] = _raise_from_template
        self._template_source = source
        self._template = environment.from_string(source) if source else None

    def _special_text(self, name: str, tokenizer_config: dict, config: dict):
        value = tokenizer_config.get(name)
        text = value.get("content") if isinstance(value, dict) else value
        if text is not None:
            return text
        key = name + "_id"
        owner = next((source for source in (tokenizer_config, config, _nested(config)) if key in source), None)
        if owner is None or owner[key] is None:
            return None
        return self._tokenizer.id_to_token(_id_tuple(owner[key], name)[0])

    @property
    def eos_token_ids(self) -> tuple[int, ...]:
        return self._eos_token_ids

    @property
    def pad_token_id(self) -> int | None:
        text = self.special.get("pad_token")
        return None if text is None else self._tokenizer.token_to_id(text)

    def _check_id(self, token_id, what: str) -> None:
        if type(token_id) is not int or token_id not in self._known_ids:
            raise ValueError(f"{what} contains an ID outside the tokenizer vocabulary: {token_id!r}")

    # -- encoding -------------------------------------------------------------------------------
    def encode_text(self, text: str, *, add_special_tokens: bool = False) -> list[int]:
        return self._tokenizer.encode(text, add_special_tokens=add_special_tokens).ids

    def _render(self, messages, *, add_generation_prompt=True, tools=None, **options) -> list[int]:
        variables = {name: text for name, text in self.special.items() if text is not None}
        try:
            text = self._template.render(messages=messages, add_generation_prompt=add_generation_prompt, tools=tools,
                                         **variables, **options)
        except (TemplateError, TypeError, ValueError) as error:
            raise ValueError(f"cannot render checkpoint chat template: {error}") from error
        ids = self.encode_text(text)
        if not ids:
            raise ValueError("chat template must produce a nonempty list of token IDs")
        return ids

    @staticmethod
    def _plain_messages(messages) -> None:
        if not isinstance(messages, list) or not messages:
            raise ValueError("messages must be a nonempty list")
        for message in messages:
            if not isinstance(message, dict) or set(message) != {"role", "content"}:
                raise ValueError("messages support only role and content")
            if message["role"] not in _ROLES:
                raise ValueError("message role must be system, user, or assistant")
            if not (isinstance(message["content"], str) and message["content"].strip()):
                raise ValueError("message content must be nonempty text")
        if messages[-1]["role"] != "user":
            raise ValueError("messages must end with a user message for generation")

    def encode_prompt(self, prompt: str | None = None, messages: list[dict] | None = None) -> list[int]:
        """Generation prompt ids for one prompt text or a chat; plain text without a template is
        tokenized with the tokenizer's own special tokens."""
        if (prompt is None) == (messages is None):
            raise ValueError("provide exactly one of prompt or messages")
        if prompt is not None:
            if not (isinstance(prompt, str) and prompt.strip()):
                raise ValueError("prompt must be a nonempty string")
            if self._template is None:
                return self.encode_text(prompt, add_special_tokens=True)
            messages = [{"role": "user", "content": prompt}]
        elif self._template is None:
            raise ValueError("messages require a checkpoint chat template")
        self._plain_messages(messages)
        return self._render(messages)

    def encode_conversation(self, messages, *, tools=None, chat_template_kwargs=None) -> list[int]:
        if self._template is None:
            raise ValueError("conversations require a checkpoint chat template")
        options = dict(chat_template_kwargs or {})
        if not set(options) <= {"enable_thinking"}:
            raise ValueError("chat_template_kwargs support only enable_thinking")
        if not (isinstance(messages, list) and messages):
            raise ValueError("messages must be a nonempty list")
        if messages[-1].get("role") not in ("user", "tool"):
            raise ValueError("conversations must end with a user message or completed tool results")
        return self._render(messages, tools=tools, **options)

    def encode_completion(self, messages, answer: str, *, chat_template_kwargs=None) -> tuple[list[int], list[int]]:
        """(generation prompt ids, ids of the conversation completed by ``answer``); the prompt must
        be a token prefix of the completed conversation."""
        if not (isinstance(answer, str) and answer.strip()):
            raise ValueError("answer must be a nonempty string")
        prompt = self.encode_conversation(messages, chat_template_kwargs=chat_template_kwargs)
        completed = self._render([*messages, {"role": "assistant", "content": answer}], add_generation_prompt=False,
                                 **(chat_template_kwargs or {}))
        if completed[:len(prompt)] != prompt:
            raise ValueError("completed conversation does not preserve the generation prompt token prefix")
        return prompt, completed

    def decode(self, ids, *, skip_special_tokens=True) -> str:
        ids = list(ids)
        for token_id in ids:
            self._check_id(token_id, "decoded token IDs")
        return self._tokenizer.decode(ids, skip_special_tokens=skip_special_tokens)


__all__ = ["ModelTokenizer", "read_eos_token_ids"]
