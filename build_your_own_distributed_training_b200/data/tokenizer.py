"""Text <-> token-id conversion for the data pipeline.

The training path never tokenizes: datasets here are token-id files, the
synthetic Markov corpus and uniform-random ids.  This module gives scripts and
data-preparation code the reference's small tokenizer surface
(``src/data/tokenizer.py``: a protocol with ``vocab_size`` / ``encode`` /
``decode``, a byte-level fallback and a HuggingFace-backed one, chosen by
``build_tokenizer(name)``), implemented independently:

* ``ByteTokenizer`` maps text to its UTF-8 bytes (ids 0..255).  ``decode``
  rejects ids outside that range instead of folding them, so a model sampling
  from a larger vocabulary is caught rather than silently mis-decoded.
* ``HFTokenizer`` loads ``transformers.AutoTokenizer`` lazily, on first use,
  so importing this module never imports ``transformers``.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable


@runtime_checkable
class Tokenizer(Protocol):
    @property
    def vocab_size(self) -> int: ...

    def encode(self, text: str) -> list[int]: ...

    def decode(self, ids: list[int]) -> str: ...


class ByteTokenizer:
    """UTF-8 bytes as token ids; needs no files and no network."""

    VOCAB = 256

    @property
    def vocab_size(self) -> int:
        return self.VOCAB

    def encode(self, text: str) -> list[int]:
        return [int(b) for b in bytearray(text, "utf-8")]

    def decode(self, ids: list[int]) -> str:
        bad = [i for i in ids if not 0 <= int(i) < self.VOCAB]
        if bad:
            raise ValueError(f"ByteTokenizer.decode: ids {bad[:8]} are outside [0, {self.VOCAB})")
        # malformed UTF-8 sequences (a cut in the middle of a character) become U+FFFD
        return bytearray(int(i) for i in ids).decode("utf-8", "replace")


class HFTokenizer:
    """A pretrained HuggingFace tokenizer (a hub name or a local directory), loaded on first use."""

    def __init__(self, name_or_path: str) -> None:
        self.name_or_path = name_or_path
        self._impl = None

    def _tok(self):
        if self._impl is None:
            try:
                import transformers
            except ImportError as exc:  # pragma: no cover - transformers is in the image
                raise ImportError(f"tokenizer {self.name_or_path!r} needs the `transformers` package; "
                                  "an empty tokenizer name selects the byte-level tokenizer") from exc
            tok = transformers.AutoTokenizer.from_pretrained(self.name_or_path)
            if getattr(tok, "pad_token_id", None) is None and getattr(tok, "eos_token", None) is not None:
                tok.pad_token = tok.eos_token  # batching code pads with end-of-sequence
            self._impl = tok
        return self._impl

    @property
    def vocab_size(self) -> int:
        return len(self._tok())

    def encode(self, text: str) -> list[int]:
        return [int(i) for i in self._tok()(text, add_special_tokens=True)["input_ids"]]

    def decode(self, ids: list[int]) -> str:
        return self._tok().decode([int(i) for i in ids])


def build_tokenizer(name_or_path: str | None) -> Tokenizer:
    """Byte-level for an empty or missing name, otherwise the named HuggingFace tokenizer."""
    if name_or_path is None or not str(name_or_path).strip():
        return ByteTokenizer()
    return HFTokenizer(str(name_or_path))
