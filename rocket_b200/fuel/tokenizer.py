"""Byte-level BPE tokenizer read from a Hugging Face ``tokenizer.json``.

    tok = Tokenizer.from_file("tokenizer.json")
    ids = tok.encode("def f(x):\\n    return x")
    text = tok.decode(ids)

Pipeline (the subset of tokenizer.json the GLM / Qwen byte-level tokenizers use):
  1. added / special tokens are split out first (longest match wins) and map to
     their ids directly;
  2. pre-tokenization: a ``Split`` regex (Unicode classes via the ``regex``
     module) and/or ``ByteLevel`` (whose own GPT-2 regex applies when
     ``use_regex`` is set), possibly inside a ``Sequence``;
  3. every piece is encoded as UTF-8 bytes and merged by the native BPE core
     (``rocket_b200._rt.BpeModel``, C++), honouring ``ignore_merges``.
Vocabulary entries are stored in the GPT-2 byte-to-unicode alphabet inside the
JSON; they are mapped back to raw bytes on load, so the native core works on
bytes only.

Behavioural counterpart of the reference's Tokenizer (engines/glm5-moe-nvfp4-2b/
src/tokenizer.h:21-45, tokenizer.cc:83-248).
"""
from __future__ import annotations

import json
import unicodedata

import regex

# GPT-2's pre-tokenizer pattern (ByteLevel with use_regex=True)
GPT2_PATTERN = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""


def bytes_to_unicode() -> dict[int, str]:
    """GPT-2's reversible byte -> printable unicode character table."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return {b: chr(c) for b, c in zip(bs, cs)}


_B2U = bytes_to_unicode()
_U2B = {u: b for b, u in _B2U.items()}


def _unbyte(s: str) -> bytes:
    return bytes(_U2B[ch] for ch in s)


class Tokenizer:
    def __init__(self, spec: dict):
        from .. import _rt
        model = spec.get("model") or {}
        if model.get("type", "BPE") != "BPE":
            raise ValueError(f"unsupported tokenizer model {model.get('type')!r} (byte-level BPE only)")
        vocab = [(_unbyte(tok), int(i)) for tok, i in model["vocab"].items()]
        merges = []
        for m in model.get("merges", []):
            a, b = m.split(" ", 1) if isinstance(m, str) else m
            merges.append((_unbyte(a), _unbyte(b)))
        self.bpe = _rt.BpeModel(vocab, merges, bool(model.get("ignore_merges", False)))
        self.added = {t["content"]: int(t["id"]) for t in spec.get("added_tokens", [])}
        self.added_by_id = {v: k for k, v in self.added.items()}
        self.special_ids = {int(t["id"]) for t in spec.get("added_tokens", []) if t.get("special")}
        self._added_re = (regex.compile("|".join(regex.escape(t) for t in sorted(self.added, key=len, reverse=True)))
                          if self.added else None)
        self._normalizer = self._build_normalizer(spec.get("normalizer"))
        self._split = self._build_pretok(spec.get("pre_tokenizer"))

    @staticmethod
    def from_file(path: str) -> "Tokenizer":
        with open(path, encoding="utf-8") as f:
            return Tokenizer(json.load(f))

    # ------------------------------------------------------------------ config
    @staticmethod
    def _build_normalizer(n):
        if n is None:
            return lambda s: s
        kind = n.get("type")
        if kind == "NFC":
            return lambda s: unicodedata.normalize("NFC", s)
        if kind == "Sequence":
            fs = [Tokenizer._build_normalizer(x) for x in n.get("normalizers", [])]

            def run(s):
                for f in fs:
                    s = f(s)
                return s
            return run
        raise ValueError(f"unsupported normalizer {kind!r}")

    @staticmethod
    def _build_pretok(p):
        """Returns a function str -> list[str] of pieces."""
        if p is None:
            return lambda s: [s] if s else []
        kind = p.get("type")
        if kind == "Sequence":
            steps = [Tokenizer._build_pretok(x) for x in p.get("pretokenizers", [])]

            def run(s):
                pieces = [s]
                for st in steps:
                    pieces = [q for piece in pieces for q in st(piece)]
                return pieces
            return run
        if kind == "ByteLevel":
            if p.get("add_prefix_space"):
                raise ValueError("ByteLevel add_prefix_space is not supported")
            if p.get("use_regex", True):
                rx = regex.compile(GPT2_PATTERN)
                return lambda s: rx.findall(s)
            return lambda s: [s] if s else []
        if kind == "Split":
            pat = p["pattern"]
            rx = regex.compile(pat["Regex"] if "Regex" in pat else regex.escape(pat["String"]))
            behavior = p.get("behavior", "Isolated")
            if p.get("invert"):
                raise ValueError("Split invert is not supported")
            if behavior != "Isolated":
                raise ValueError(f"Split behavior {behavior!r} is not supported")

            def split(s):
                out, last = [], 0
                for m in rx.finditer(s):
                    if m.start() > last:
                        out.append(s[last:m.start()])
                    if m.end() > m.start():
                        out.append(m.group(0))
                    last = m.end()
                if last < len(s):
                    out.append(s[last:])
                return out
            return split
        if kind == "Digits":
            rx = regex.compile(r"\p{N}" if p.get("individual_digits") else r"\p{N}+")

            def digits(s):
                out, last = [], 0
                for m in rx.finditer(s):
                    if m.start() > last:
                        out.append(s[last:m.start()])
                    out.append(m.group(0))
                    last = m.end()
                if last < len(s):
                    out.append(s[last:])
                return out
            return digits
        raise ValueError(f"unsupported pre_tokenizer {kind!r}")

    # ------------------------------------------------------------------ API
    def encode(self, text: str, allow_special: bool = True) -> list[int]:
        ids: list[int] = []
        segments = [(text, False)]
        if allow_special and self._added_re is not None:
            segments, last = [], 0
            for m in self._added_re.finditer(text):
                if m.start() > last:
                    segments.append((text[last:m.start()], False))
                segments.append((m.group(0), True))
                last = m.end()
            if last < len(text):
                segments.append((text[last:], False))
        for seg, is_added in segments:
            if is_added:
                ids.append(self.added[seg])
                continue
            pieces = self._split(self._normalizer(seg))
            ids.extend(self.bpe.encode_pieces([p.encode("utf-8") for p in pieces]))
        return ids

    def decode(self, ids, skip_special: bool = False) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i in self.added_by_id:
                if not (skip_special and i in self.special_ids):
                    out += self.added_by_id[i].encode("utf-8")
                continue
            out += self.bpe.decode([i])
        return out.decode("utf-8", errors="replace")

    @property
    def vocab_size(self) -> int:
        return max(self.bpe.vocab_size(), max(self.added_by_id, default=-1) + 1)
