"""Tokenizer protocol with a HuggingFace-backed and a byte-level implementation
(``src/data/tokenizer.py:23-91``).  ``build_tokenizer("")`` gives bytes."""

from __future__ import annotations

from typing import Protocol


class Tokenizer(Protocol):
    @property
    def vocab_size(self) -> int: ...

    def encode(self, text: str) -> list[int]: ...

    def decode(self, ids: list[int]) -> str: ...


class HFTokenizer:
    def __init__(self, name_or_path: str) -> None:
        try:
            from transformers import AutoTokenizer
        except ImportError as exc:  # pragma: no cover
            raise ImportError("HFTokenizer needs `transformers`; use ByteTokenizer otherwise.") from exc
        self._tok = AutoTokenizer.from_pretrained(name_or_path)
        if self._tok.pad_token is None:
            self._tok.pad_token = self._tok.eos_token

    @property
    def vocab_size(self) -> int:
        return int(self._tok.vocab_size)

    def encode(self, text: str) -> list[int]:
        return list(self._tok.encode(text))

    def decode(self, ids: list[int]) -> str:
        return str(self._tok.decode(ids))


class ByteTokenizer:
    @property
    def vocab_size(self) -> int:
        return 256

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: list[int]) -> str:
        return bytes(i % 256 for i in ids).decode("utf-8", errors="replace")


def build_tokenizer(name_or_path: str | None) -> Tokenizer:
    return ByteTokenizer() if not name_or_path else HFTokenizer(name_or_path)
