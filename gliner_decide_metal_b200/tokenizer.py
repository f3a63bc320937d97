"""Native tokenizer and GLiNER classification-schema formatter
(``NativeDecisionTokenizer``, NativeTokenizer.swift:55-264).

The reference loads the checkpoint's ``tokenizer.json`` (a Hugging Face tokenizers file:
DeBERTa-v3's SentencePiece Unigram model) through swift-transformers and formats each
request as GLiNER2's classification schema:

* per task ``( [P] <name[: prompt]>[ [DESCRIPTION] label: text ...] ( [L] label ... ) )``,
  tasks joined by ``[SEP_STRUCT]``, then ``[SEP_TEXT]`` and the text's words
  (NativeTokenizer.swift:90-120);
* the text gets a ``.`` unless it already ends in ``.``, ``!`` or ``?`` (``.`` when empty),
  is split by the reference's word regex and lower-cased (:198-212);
* every entry is tokenised on its own: occurrences of the file's added tokens become their
  ids (earliest match first, the longest on ties), the rest goes through the Unigram model
  (:160-196); the position of each ``[L]`` entry's first id is its label marker (:127-133);
* the ids go to the smallest bucket that holds them, with ``[PAD]`` padding and the marker
  layout [1, Hm, O] (:134-157; here ``make_input_from_tokens`` over ``gdc_layout_row``).

The Unigram part (``UnigramTokenizer``) follows the tokenizers-library algorithm the file
format defines: the normalizer and pre-tokenizer chain of the file, then a Viterbi search
for the segmentation with the largest sum of piece scores; a character no piece covers
becomes an unknown node scored ``min(score) - 10``, and runs of unknown nodes fuse into one
``unk_id``. ``Precompiled`` normalizers (a SentencePiece character map, DeBERTa-v3's
``nmt_nfkc``) are applied from the map itself: its double-array trie is searched per
extended grapheme cluster as the tokenizers library does. The checkpoint's own
``tokenizer.json`` is not available here; tests pin this implementation to the tokenizers
library on synthetic vocabularies and on a SentencePiece ``nmt_nfkc`` model trained in the
test.
"""
from __future__ import annotations

import base64
import json
import re
import struct
import unicodedata
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

import regex


from . import DEFAULT_BUCKETS, DecisionInput, DecisionTask, NoTaskLabelsError, make_input_from_tokens

_UNK_PENALTY = 10.0


class TokenizerFilesError(FileNotFoundError):
    """``NativeTokenizerError.missingTokenizerFiles`` (NativeTokenizer.swift:6,233-237)."""


# --------------------------------------------------------------------------- normalizers

class PrecompiledCharsMap:
    """A SentencePiece precompiled character map: a little-endian uint32 trie size, a
    darts-clone double-array trie over UTF-8 keys (uint32 units), then the replacement
    strings, each NUL-terminated; a key's value is the offset of its replacement.

    ``normalize`` follows the tokenizers library's ``Precompiled`` normalizer: per extended
    grapheme cluster, a cluster shorter than 6 bytes is replaced by the replacement of its
    first (shortest) key prefix if it has one; otherwise each character is replaced by its
    own, or kept."""

    def __init__(self, blob: bytes):
        (trie_size,) = struct.unpack_from("<I", blob, 0)
        self.units = struct.unpack_from(f"<{trie_size // 4}I", blob, 4)
        self.strings = blob[4 + trie_size:]
        self._memo: Dict[str, Optional[str]] = {}

    def _first_prefix(self, key: bytes) -> Optional[int]:
        # darts-clone unit fields: has_leaf = bit 8, value = low 31 bits (leaf units),
        # label = low 8 bits plus bit 31, offset = (unit >> 10) << ((unit & 0x200) >> 6)
        units = self.units
        pos = 0
        unit = units[pos]
        pos ^= (unit >> 10) << ((unit & 0x200) >> 6)
        for c in key:
            pos ^= c
            if pos >= len(units):
                return None
            unit = units[pos]
            if (unit & 0x800000FF) != c:
                return None
            pos ^= (unit >> 10) << ((unit & 0x200) >> 6)
            if (unit >> 8) & 1:
                return units[pos] & 0x7FFFFFFF
        return None

    def transform(self, chunk: str) -> Optional[str]:
        hit = self._memo.get(chunk, False)
        if hit is not False:
            return hit
        off = self._first_prefix(chunk.encode("utf-8"))
        out = None
        if off is not None:
            end = self.strings.find(b"\0", off)
            out = self.strings[off:end if end >= 0 else len(self.strings)].decode("utf-8", errors="replace")
        self._memo[chunk] = out
        return out

    def normalize(self, s: str) -> str:
        import regex  # extended grapheme clusters (\X)
        out = []
        for g in regex.findall(r"\X", s):
            if len(g.encode("utf-8")) < 6:
                n = self.transform(g)
                if n is not None:
                    out.append(n)
                    continue
            for ch in g:
                n = self.transform(ch)
                out.append(ch if n is None else n)
        return "".join(out)


def _normalizer(spec: Optional[dict]):
    """Callable str -> str for a tokenizers ``normalizer`` entry."""
    if spec is None:
        return lambda s: s
    kind = spec.get("type")
    if kind == "Sequence":
        parts = [_normalizer(x) for x in spec.get("normalizers", [])]

        def seq(s):
            for p in parts:
                s = p(s)
            return s
        return seq
    if kind in ("NFKC", "NFC", "NFD", "NFKD"):
        return lambda s: unicodedata.normalize(kind, s)
    if kind == "Precompiled":
        blob = spec.get("precompiled_charsmap")
        if not blob:
            return lambda s: s
        cmap = PrecompiledCharsMap(base64.b64decode(blob))
        return cmap.normalize
    if kind == "Lowercase":
        return lambda s: s.lower()
    if kind == "Strip":
        left, right = spec.get("strip_left", True), spec.get("strip_right", True)

        def strip(s):
            if left:
                s = s.lstrip()
            if right:
                s = s.rstrip()
            return s
        return strip
    if kind == "Replace":
        pat, content = spec["pattern"], spec.get("content", "")
        if "Regex" in pat:
            rx = re.compile(pat["Regex"])
            return lambda s: rx.sub(lambda _m: content, s)
        lit = pat["String"]
        return lambda s: s.replace(lit, content)
    raise ValueError(f"unsupported normalizer {kind!r}")


# --------------------------------------------------------------------------- pre-tokenizers

def _pre_tokenizer(spec: Optional[dict]):
    """Callable str -> list[str] for a tokenizers ``pre_tokenizer`` entry."""
    if spec is None:
        return lambda s: [s] if s else []
    kind = spec.get("type")
    if kind == "Sequence":
        parts = [_pre_tokenizer(x) for x in spec.get("pretokenizers", [])]

        def seq(s):
            pieces = [s]
            for p in parts:
                pieces = [q for piece in pieces for q in p(piece)]
            return pieces
        return seq
    if kind == "Metaspace":
        # prepend_scheme "first" is applied like "always" (one call sees one text); the
        # tokenizers library also skips the prefix when a normalizer removed leading text,
        # which DeBERTa-v3's "always" never does
        rep = spec.get("replacement", "▁")
        scheme = spec.get("prepend_scheme", "always" if spec.get("add_prefix_space", True) else "never")
        split = spec.get("split", True)

        def metaspace(s):
            if not s:
                return []
            s = s.replace(" ", rep)
            if scheme in ("always", "first") and not s.startswith(rep):
                s = rep + s
            if not split:
                return [s] if s else []
            out, start = [], 0
            for i in range(1, len(s)):
                if s[i] == rep:
                    out.append(s[start:i])
                    start = i
            if s:
                out.append(s[start:])
            return out
        return metaspace
    if kind == "WhitespaceSplit":
        return lambda s: s.split()
    if kind == "Punctuation":
        def punct(s):
            out, cur = [], ""
            for ch in s:
                if unicodedata.category(ch).startswith("P"):
                    if cur:
                        out.append(cur)
                    out.append(ch)
                    cur = ""
                else:
                    cur += ch
            if cur:
                out.append(cur)
            return out
        return punct
    raise ValueError(f"unsupported pre-tokenizer {kind!r}")


# --------------------------------------------------------------------------- Unigram

class UnigramTokenizer:
    """A tokenizers-format Unigram model with its normalizer and pre-tokenizer."""

    def __init__(self, spec: dict):
        model = spec.get("model") or {}
        if model.get("type") != "Unigram":
            raise ValueError(f"expected a Unigram model, got {model.get('type')!r}")
        if model.get("byte_fallback"):
            raise ValueError("byte_fallback Unigram models are not supported")
        vocab = model["vocab"]
        self.unk_id: Optional[int] = model.get("unk_id")
        self.pieces: Dict[str, Tuple[int, float]] = {}
        for i, (piece, score) in enumerate(vocab):
            self.pieces.setdefault(piece, (i, float(score)))
        self.max_len = max((len(p) for p in self.pieces), default=1)
        self.unk_score = min((s for _, s in self.pieces.values()), default=0.0) - _UNK_PENALTY
        self.added: Dict[str, int] = {t["content"]: int(t["id"]) for t in spec.get("added_tokens", [])}
        self.normalize = _normalizer(spec.get("normalizer"))
        self.pre_tokenize = _pre_tokenizer(spec.get("pre_tokenizer"))

    @staticmethod
    def from_file(path) -> "UnigramTokenizer":
        with open(path, "r", encoding="utf-8") as f:
            return UnigramTokenizer(json.load(f))

    def _viterbi(self, s: str) -> List[Tuple[str, Optional[int]]]:
        """Best segmentation of one pre-token: (surface, id or None for unknown)."""
        n = len(s)
        best = [float("-inf")] * (n + 1)
        back: List[Optional[Tuple[int, Optional[int]]]] = [None] * (n + 1)
        best[0] = 0.0
        for b in range(n):
            if best[b] == float("-inf"):
                continue
            single = False
            for e in range(b + 1, min(n, b + self.max_len) + 1):
                hit = self.pieces.get(s[b:e])
                if hit is None:
                    continue
                if e == b + 1:
                    single = True
                sc = best[b] + hit[1]
                if sc > best[e]:
                    best[e], back[e] = sc, (b, hit[0])
            if not single:
                sc = best[b] + self.unk_score
                if sc > best[b + 1]:
                    best[b + 1], back[b + 1] = sc, (b, None)
        out: List[Tuple[str, Optional[int]]] = []
        e = n
        while e > 0:
            b, tid = back[e]
            out.append((s[b:e], tid))
            e = b
        out.reverse()
        fused: List[Tuple[str, Optional[int]]] = []
        for surf, tid in out:  # consecutive unknown pieces become one
            if tid is None and fused and fused[-1][1] is None:
                fused[-1] = (fused[-1][0] + surf, None)
            else:
                fused.append((surf, tid))
        return fused

    def tokenize(self, text: str) -> List[str]:
        """Surface pieces (unknown runs as their text), like ``Tokenizer.encode(...).tokens``."""
        return [surf for surf, _ in self._encode(text)]

    def encode(self, text: str) -> List[int]:
        """Piece ids; unknown runs map to ``unk_id`` (or 0 without one)."""
        unk = self.unk_id if self.unk_id is not None else 0
        return [unk if tid is None else tid for _, tid in self._encode(text)]

    def _encode(self, text: str):
        out = []
        for pre in self.pre_tokenize(self.normalize(text)):
            out.extend(self._viterbi(pre))
        return out


# --------------------------------------------------------------------------- schema formatter

# NativeTokenizer.swift:67-71: NSRegularExpression (ICU) with .caseInsensitive. The classes
# are spelled out as ICU defines them, because Python's re module differs on non-ASCII text:
#   ICU \w = [\p{Alphabetic}\p{Mark}\p{Decimal_Number}\p{Connector_Punctuation}\u200c\u200d]
#         (re's \w misses combining marks, ZWNJ / ZWJ, Other_Alphabetic symbols such as circled
#         letters and connector punctuation other than "_", and adds non-decimal numbers such as
#         superscripts and fractions)
#   ICU \s = [\t\n\f\r\p{Z}] (re's \s also takes \v, U+001C-U+001F and U+0085)
#   case-insensitive ASCII letters: simple case folding adds U+017F (long s) to s and U+212A
#         (Kelvin sign) to k; nothing else folds to an ASCII letter.
_ICU_W = r"[\p{Alphabetic}\p{Mark}\p{Nd}\p{Pc}\u200c\u200d]"
_ICU_SPACE = r"\t\n\f\r\p{Z}"
_LETTERS = r"a-zA-Z\u017f\u212a"


def _ci(word: str) -> str:
    """A literal ASCII word matched case-insensitively, one class per letter."""
    extra = {"s": "\u017f", "k": "\u212a"}
    return "".join(f"[{c}{c.upper()}{extra.get(c, '')}]" if c.isalpha() else regex.escape(c) for c in word)


_WORD_RE = regex.compile(
    rf"(?:{_ci('http')}{_ci('s')}?://[^{_ICU_SPACE}]+|{_ci('www.')}[^{_ICU_SPACE}]+)"
    rf"|[{_LETTERS}0-9._%+-]+@[{_LETTERS}0-9.-]+\.[{_LETTERS}]{{2,}}"
    rf"|@[{_LETTERS}0-9_]+"
    rf"|{_ICU_W}+(?:[-_]{_ICU_W}+)*"
    rf"|[^{_ICU_SPACE}]",
    regex.VERSION0)


def split_words(text: str) -> List[str]:
    """Sentence-final punctuation, word split and lower-casing (NativeTokenizer.swift:198-212)."""
    if not text:
        norm = "."
    elif text[-1] in ".!?":
        norm = text
    else:
        norm = text + "."
    return [m.group(0).lower() for m in _WORD_RE.finditer(norm)]


@dataclass
class _Entry:
    text: str
    label_of: Optional[int] = None  # task index of an [L] entry


def schema_entries(text: str, tasks: Sequence[DecisionTask]) -> List[_Entry]:
    """The classification schema of NativeTokenizer.swift:90-120, one entry per piece of text."""
    out: List[_Entry] = []
    for ti, task in enumerate(tasks):
        prompt = f"{task.name}: {task.prompt}" if task.prompt is not None else task.name
        desc = "".join(f" [DESCRIPTION] {lab}: {task.label_descriptions[lab]}"
                       for lab in task.labels if task.label_descriptions and lab in task.label_descriptions)
        out += [_Entry("("), _Entry("[P]"), _Entry(prompt + desc), _Entry("(")]
        for lab in task.labels:
            out += [_Entry("[L]", ti), _Entry(lab)]
        out += [_Entry(")"), _Entry(")")]
        if ti < len(tasks) - 1:
            out.append(_Entry("[SEP_STRUCT]"))
    out.append(_Entry("[SEP_TEXT]"))
    out += [_Entry(w) for w in split_words(text)]
    return out


class NativeDecisionTokenizer:
    """``NativeDecisionTokenizer(directory:)`` (NativeTokenizer.swift:59-74): the directory
    holds ``tokenizer.json`` and ``tokenizer_config.json``."""

    def __init__(self, directory):
        d = Path(directory)
        if not (d / "tokenizer.json").is_file() or not (d / "tokenizer_config.json").is_file():
            raise TokenizerFilesError(f"Tokenizer directory is missing tokenizer.json/tokenizer_config.json: {d}")
        self.unigram = UnigramTokenizer.from_file(d / "tokenizer.json")
        self.special = dict(self.unigram.added)
        # Each schema entry (one word of the text, a label, a prompt) is tokenised on its own,
        # so its ids depend on the entry alone: they are cached (bounded) for the repeated
        # words of real text.
        self._cache: Dict[str, List[int]] = {}
        # earliest match first; at one position the alternation tries longer tokens first
        self._special_rx = (re.compile("|".join(re.escape(t) for t in sorted(self.special, key=len, reverse=True)))
                            if self.special else None)
        self.pad_id = self.special.get("[PAD]", self.unigram.pieces.get("[PAD]", (0, 0.0))[0])

    def token_ids(self, text: str) -> List[int]:
        """Ids of one schema entry: added tokens matched first (earliest, then longest),
        the text between them through the Unigram model (NativeTokenizer.swift:160-196)."""
        hit = self._cache.get(text)
        if hit is not None:
            return hit
        ids: List[int] = []
        cur = 0
        while cur < len(text):
            m = self._special_rx.search(text, cur) if self._special_rx is not None else None
            if m is None:
                ids += self._plain(text[cur:])
                break
            if m.start() > cur:
                ids += self._plain(text[cur:m.start()])
            ids.append(self.special[m.group(0)])
            cur = m.end()
        if len(self._cache) >= 200_000:
            self._cache.clear()
        self._cache[text] = ids
        return ids

    def _plain(self, text: str) -> List[int]:
        return self.unigram.encode(text)

    def encode_schema(self, text: str, tasks: Sequence[DecisionTask]) -> Tuple[List[int], List[List[int]]]:
        """Unpadded ids and, per task, the positions of its label markers."""
        if not tasks or any(len(t.labels) == 0 for t in tasks):
            raise NoTaskLabelsError(5, "Every decision task must contain at least one label")
        ids: List[int] = []
        markers: List[List[int]] = [[] for _ in tasks]
        for entry in schema_entries(text, tasks):
            start = len(ids)
            ids.extend(self.token_ids(entry.text))
            if entry.label_of is not None:
                markers[entry.label_of].append(start)
        return ids, markers

    def make_input(self, text: str, tasks: Sequence[DecisionTask], buckets=DEFAULT_BUCKETS) -> DecisionInput:
        """``makeInput(text:tasks:buckets:)`` (NativeTokenizer.swift:76-158)."""
        ids, markers = self.encode_schema(text, tasks)
        return make_input_from_tokens(ids, markers, buckets, pad_id=self.pad_id)
