"""Prompts for the AR loop: the text/ABC tokenizer and the token layout of each phase.

What the AR engine is fed upstream of ``yar_generate``: ``Pipeline::generate`` builds the
conditional and unconditional prefixes from a song request with the checkpoint's text
tokenizer (native/src/protocol.mm:322-360, vendor/yue/src/yue2/protocol.py:95-141) and
hands them to ``generate_tokens``. This module restates that layer:

* ``TextTokenizer`` — the frozen byte-level BPE (protocol.mm:428-592,
  tokenization_yue2.py:8-31): ``qwen.tiktoken`` lines of ``base64(token) rank`` give the
  151,643 ordinary tokens; text is NFC-normalized, split by the pre-tokenizer pattern
  ``PATTERN`` into pieces, and each piece's bytes are merged pairwise, always the adjacent
  pair whose concatenation has the lowest rank (leftmost on ties), until no adjacent pair
  is a token; the 208 special and extra tokens follow the ordinary ones (ids 151643..).
  Upstream runs this through tiktoken (Python) or its own priority-queue merge (C++); the
  merge rule is the published byte-pair encoding, written here from that rule.
* ``SongRequest`` / ``token_prefixes`` / ``negative_prefix`` / ``chunk_ranges`` — the
  prompt layout and its validation (protocol.py:73-141).

The instruction strings, the special-token ids and the pre-tokenizer pattern are the
checkpoint's protocol: they must be the reference's exactly for the model to see the
prompts it was trained on.
"""
from __future__ import annotations

import base64
import math
import re
import unicodedata
from dataclasses import asdict, dataclass

EOD = 151643
ABC_START, ABC_END = 151847, 151848
MUSIC_START, MUSIC_END = 151851, 151852
CODEC_OFFSET, CODEC_SIZE = 151853, 32768
VOCAB_SIZE, CONTEXT = 184704, 24576
PROTOCOL_VERSION = "yue2-native-v1"

INSTRUCTIONS = {
    "off": "Generate music with codec tokens from the given conditions.",
    "melody": "Generate a melody-only ABC transcription without chord symbols, then generate music with codec "
              "tokens from the given conditions.",
    "full": "Generate a chord-annotated ABC transcription, then generate music with codec tokens from the given "
            "conditions.",
}

# Pre-tokenizer (protocol.mm:475-481, tokenization_yue2.py:18): contractions, letter runs
# with one optional leading non-letter, single digits, punctuation runs, newlines, spaces.
PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+"
           r"|\s+(?!\S)|\s+")

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<R>", "<S>", "<X>", "<mask>", "<sep>"] + \
           [f"<extra_{i}>" for i in range(200)]
SPECIALS[ABC_START - EOD] = "<abc>"
SPECIALS[ABC_END - EOD] = "</abc>"


def _regex():
    try:
        import regex  # \p{L} / \p{N} classes, which the standard library's re lacks
    except ImportError as e:  # pragma: no cover - the image ships it
        raise RuntimeError("the tokenizer needs the 'regex' package for Unicode classes") from e
    return regex.compile(PATTERN)


class TextTokenizer:
    """The checkpoint's text / ABC tokenizer (``qwen.tiktoken``)."""

    def __init__(self, path: str, ordinary: int = EOD):
        ranks: dict[bytes, int] = {}
        with open(path, "rb") as f:
            for line in f.read().splitlines():
                if not line:
                    continue
                parts = line.split()
                if len(parts) != 2:
                    raise ValueError("Invalid checkpoint-native qwen.tiktoken vocabulary")
                try:
                    token, rank = base64.b64decode(parts[0], validate=True), int(parts[1])
                except ValueError as e:
                    raise ValueError("Invalid base64 vocabulary token") from e
                if not token or not 0 <= rank < ordinary:
                    raise ValueError("Invalid checkpoint-native qwen.tiktoken vocabulary")
                ranks[token] = rank
        if len(ranks) != ordinary or len(set(ranks.values())) != ordinary:
            raise ValueError(f"Expected checkpoint-native qwen.tiktoken ({ordinary} ordinary tokens)")
        self.ranks = ranks
        self.pieces = [b""] * ordinary
        for token, rank in ranks.items():
            self.pieces[rank] = token
        self.specials = [s.encode() for s in SPECIALS]
        self._split = _regex()

    @property
    def n_vocab(self) -> int:
        return len(self.pieces) + len(self.specials)

    def _bpe(self, piece: bytes, out: list[int]) -> None:
        direct = self.ranks.get(piece)
        if direct is not None:
            out.append(direct)
            return
        parts = [piece[i:i + 1] for i in range(len(piece))]
        while len(parts) > 1:
            best, at = None, -1
            for i in range(len(parts) - 1):
                r = self.ranks.get(parts[i] + parts[i + 1])
                if r is not None and (best is None or r < best):
                    best, at = r, i
            if best is None:
                break
            parts[at:at + 2] = [parts[at] + parts[at + 1]]
        for p in parts:
            r = self.ranks.get(p)
            if r is None:
                raise ValueError("Vocabulary is missing a byte token")
            out.append(r)

    def encode(self, text: str) -> list[int]:
        """Ordinary tokens of ``text`` (special-token text is encoded as plain text)."""
        normalized = unicodedata.normalize("NFC", text)
        out: list[int] = []
        pos = 0
        for m in self._split.finditer(normalized):
            if m.start() != pos or m.end() == m.start():
                raise RuntimeError("Tokenizer regex did not cover input")
            self._bpe(m.group().encode("utf-8"), out)
            pos = m.end()
        if pos != len(normalized):
            raise RuntimeError("Tokenizer regex did not cover input")
        return out

    def decode(self, ids) -> str:
        """Text of ``ids``; ids outside the vocabulary are skipped, bad UTF-8 replaced."""
        raw = b"".join(self.pieces[i] if i < len(self.pieces) else self.specials[i - len(self.pieces)]
                       for i in (int(t) for t in ids) if 0 <= i < self.n_vocab)
        return raw.decode("utf-8", errors="replace")


@dataclass(frozen=True)
class SongRequest:
    """A song's conditions (protocol.py:73-107): style tags, lyrics, the ABC mode `cot`
    (off / melody / full), seed, optional external ABC text and CFG scale, and an id."""
    style: str
    lyrics: str
    cot: str = "full"
    seed: int = 831001
    abc: str | None = None
    cfg_scale: float | None = None
    id: str = "song"

    def __post_init__(self):
        if self.cot not in INSTRUCTIONS:
            raise ValueError("cot must be off, melody or full")
        if not isinstance(self.style, str) or not isinstance(self.lyrics, str):
            raise TypeError("style and lyrics must be strings")
        if type(self.seed) is not int or not 0 <= self.seed < 2 ** 63:
            raise ValueError("seed must be an integer in [0, 2**63)")
        if not re.fullmatch(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,179}", self.id) or self.id in {".", ".."}:
            raise ValueError("id must be a filename-safe identifier")
        if self.abc is not None and (self.cot == "off" or not isinstance(self.abc, str) or not self.abc.strip()):
            raise ValueError("External ABC requires nonempty text and cot=melody/full")
        if self.cfg_scale is not None and (not math.isfinite(self.cfg_scale) or not 0 <= self.cfg_scale <= 20):
            raise ValueError("cfg_scale must be finite and in [0,20]")

    @property
    def guidance(self) -> float:
        """The semantic phase's CFG scale: 1.01 for cot=off, 1.0 otherwise, unless given."""
        return (1.01 if self.cot == "off" else 1.0) if self.cfg_scale is None else self.cfg_scale

    def text(self) -> str:
        return f"{INSTRUCTIONS[self.cot]}\n[Tags]\n{self.style}\n[Lyrics]\n{self.lyrics}\n"

    def to_dict(self) -> dict:
        return asdict(self)


def _check_abc(ids) -> list[int]:
    ids = list(ids)
    if any(type(t) is not int or not 0 <= t < EOD for t in ids):
        raise ValueError("ABC IDs must remain inside the ordinary text vocabulary")
    return ids


def token_prefixes(request: SongRequest, tokenizer: TextTokenizer, abc_ids=None) -> list[int]:
    """The conditional prefix: EOD, the request text, then for cot=off the empty ABC block
    and MUSIC_START (the semantic phase starts at once); otherwise ABC_START alone (the ABC
    phase generates the transcription) or, with ABC ids given or external ABC text, the
    whole block and MUSIC_START."""
    base = [EOD] + tokenizer.encode(request.text())
    if request.cot == "off":
        return base + [ABC_START, ABC_END, MUSIC_START]
    if abc_ids is None:
        if request.abc is None:
            return base + [ABC_START]
        abc_ids = tokenizer.encode(request.abc)
    return base + [ABC_START] + _check_abc(abc_ids) + [ABC_END, MUSIC_START]


def negative_prefix(request: SongRequest, tokenizer: TextTokenizer, abc_ids=None) -> list[int]:
    """The unconditional prefix of the semantic phase's CFG: the instruction alone (no
    style or lyrics), and for cot=melody/full the positive branch's exact ABC ids."""
    base = [EOD] + tokenizer.encode(INSTRUCTIONS[request.cot])
    if request.cot == "off":
        return base + [MUSIC_START]
    if abc_ids is None:
        raise ValueError("Symbolic CFG must retain the exact positive-branch ABC IDs")
    return base + [ABC_START] + _check_abc(abc_ids) + [ABC_END, MUSIC_START]


def chunk_ranges(frames: int, prefix_tokens: int, context: int = CONTEXT) -> list[tuple[int, int]]:
    """Codec-frame ranges the acoustic stage conditions on per chunk (protocol.py:144-148)."""
    size = min((context - prefix_tokens - 3) // 2, CONTEXT)
    if frames < 1 or size < 1:
        raise ValueError("Empty codec or prefix leaves no acoustic context")
    return [(a, min(a + size, frames)) for a in range(0, frames, size)]
