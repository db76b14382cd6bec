"""Qwen tokenizer: ChatML encode and streaming UTF-8 decode over a byte-level
BPE read from a Hugging Face `tokenizer.json`.

Mirrors QwenTokenizer (QwenTokenizer.swift:11-70) and formatPrompt
(main.swift:11-13).  The reference delegates the BPE to swift-transformers
(`AutoTokenizer.from(modelFolder:)`, QwenTokenizer.swift:17-24); this module
implements the same published algorithm from the file's own tables:

  * added tokens are matched in the raw text first (longest content first);
  * the rest is NFC-normalised (when the file's normalizer says so), split by
    the file's pre-tokenizer regex (each match and each gap is a piece), and
    each piece's UTF-8 bytes are mapped to printable characters (the byte-level
    table of GPT-2: printable Latin-1 bytes map to themselves, the others to
    U+0100 onwards in byte order);
  * a piece is merged by BPE: repeatedly the adjacent pair with the lowest
    merge rank is joined (every occurrence, left to right), then the symbols
    are looked up in the vocabulary;
  * decoding maps byte-level symbols back to bytes, keeps added tokens' text,
    and decodes UTF-8 with U+FFFD for incomplete sequences.

QwenTokenizer.encode splits the ChatML tags itself (<|im_start|> = 151644,
<|im_end|> = 151645, QwenTokenizer.swift:26-50); decode keeps a rolling buffer
and returns "" while the buffer still decodes to a replacement character
(:52-69).
"""
from __future__ import annotations

import json
import os
import unicodedata

IM_START, IM_END = 151644, 151645


def format_prompt(user_query: str) -> str:
    """main.swift:11-13."""
    return ("<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n<|im_start|>user\n"
            f"{user_query}<|im_end|>\n<|im_start|>assistant\n")


def byte_level_table() -> dict:
    """byte -> printable character of the byte-level BPE."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


class BPETokenizer:
    """Byte-level BPE from a tokenizer.json (model type BPE)."""

    def __init__(self, path: str):
        import regex

        with open(path, encoding="utf-8") as f:
            cfg = json.load(f)
        model = cfg["model"]
        if model.get("type", "BPE") != "BPE":
            raise ValueError(f"{path}: model type {model.get('type')} is not BPE")
        self.vocab = dict(model["vocab"])
        merges = model.get("merges", [])
        self.ranks = {}
        for r, m in enumerate(merges):
            a, b = (m.split(" ", 1) if isinstance(m, str) else m)
            self.ranks[(a, b)] = r
        self.added = {t["content"]: t["id"] for t in cfg.get("added_tokens", [])}
        self.id_to_token = {i: t for t, i in self.vocab.items()}
        self.added_by_id = {i: t for t, i in self.added.items()}
        norm = cfg.get("normalizer") or {}
        kinds = [n.get("type") for n in norm.get("normalizers", [norm])] if norm else []
        self.nfc = "NFC" in kinds
        pattern = None
        pre = cfg.get("pre_tokenizer") or {}
        for p in pre.get("pretokenizers", [pre]) if pre else []:
            if p.get("type") == "Split":
                pattern = p["pattern"].get("Regex") or regex.escape(p["pattern"].get("String", ""))
            elif p.get("type") == "ByteLevel" and p.get("use_regex", True) and pattern is None:
                pattern = (r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+")
        self.split = regex.compile(pattern) if pattern else None
        self.added_split = (regex.compile("|".join(regex.escape(t) for t in
                                                   sorted(self.added, key=len, reverse=True)))
                            if self.added else None)
        self.b2c = byte_level_table()
        self.c2b = {c: b for b, c in self.b2c.items()}
        self.cache = {}

    # -- encode -------------------------------------------------------------
    def _pieces(self, text: str):
        if self.nfc:
            text = unicodedata.normalize("NFC", text)
        if self.split is None:
            yield text
            return
        pos = 0
        for m in self.split.finditer(text):
            if m.start() > pos:
                yield text[pos:m.start()]
            if m.end() > m.start():
                yield m.group(0)
            pos = m.end()
        if pos < len(text):
            yield text[pos:]

    def _bpe(self, piece: str) -> list:
        hit = self.cache.get(piece)
        if hit is not None:
            return hit
        syms = [self.b2c[b] for b in piece.encode("utf-8")]
        while len(syms) > 1:
            best, best_rank = None, None
            for pair in zip(syms, syms[1:]):
                r = self.ranks.get(pair)
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = pair, r
            if best is None:
                break
            out, i = [], 0
            while i < len(syms):
                if i + 1 < len(syms) and (syms[i], syms[i + 1]) == best:
                    out.append(syms[i] + syms[i + 1])
                    i += 2
                else:
                    out.append(syms[i])
                    i += 1
            syms = out
        ids = []
        for s in syms:
            if s not in self.vocab:
                raise KeyError(f"symbol {s!r} is not in the vocabulary")
            ids.append(self.vocab[s])
        if len(self.cache) < 1 << 16:
            self.cache[piece] = ids
        return ids

    def encode(self, text: str) -> list:
        ids, pos = [], 0
        segments = []
        if self.added_split is not None:
            for m in self.added_split.finditer(text):
                segments.append((text[pos:m.start()], None))
                segments.append((None, self.added[m.group(0)]))
                pos = m.end()
        segments.append((text[pos:], None))
        for seg, tok in segments:
            if tok is not None:
                ids.append(tok)
            elif seg:
                for piece in self._pieces(seg):
                    ids.extend(self._bpe(piece))
        return ids

    # -- decode -------------------------------------------------------------
    def decode_bytes(self, ids) -> bytes:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i in self.added_by_id:
                out += self.added_by_id[i].encode("utf-8")
                continue
            tok = self.id_to_token.get(i)
            if tok is None:
                raise KeyError(f"token id {i} is not in the vocabulary")
            for ch in tok:
                b = self.c2b.get(ch)
                if b is None:
                    out += ch.encode("utf-8")
                else:
                    out.append(b)
        return bytes(out)

    def decode(self, ids) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")


class QwenTokenizer:
    """QwenTokenizer.swift: tokenizer.json from the weights directory."""

    def __init__(self, weights_dir: str):
        path = os.path.join(weights_dir, "tokenizer.json")
        if not os.path.exists(path):
            raise FileNotFoundError(f"Tokenizer weights file not found at {path}")
        self.tokenizer = BPETokenizer(path)
        self._buffer = []

    def encode(self, prompt: str) -> list:
        """ChatML tags by hand, the text between them by the BPE (:26-50)."""
        tokens = []
        for i, start_part in enumerate(prompt.split("<|im_start|>")):
            if i > 0:
                tokens.append(IM_START)
            for j, end_part in enumerate(start_part.split("<|im_end|>")):
                if j > 0:
                    tokens.append(IM_END)
                if end_part:
                    tokens.extend(self.tokenizer.encode(end_part))
        return tokens

    def decode(self, tokens) -> str:
        """Rolling buffer: "" while the buffered tokens end inside a UTF-8
        sequence, else the buffered text (and the buffer is cleared) (:52-69)."""
        self._buffer.extend(int(t) for t in tokens)
        text = self.tokenizer.decode(self._buffer)
        if "�" in text:
            return ""
        self._buffer.clear()
        return text


def stream_generate(forward, tokenizer: QwenTokenizer, prompt: str, max_tokens: int = 64,
                    write=None) -> str:
    """generate(prompt:maxTokens:) (InferenceEngine.swift:29-52) over any
    forward(token_id, position) -> next id: the ChatML-encoded prompt is fed one
    position at a time, then up to max_tokens sampled tokens are decoded and
    written as their text completes, stopping at <|im_end|> (151645) or
    <|endoftext|> (151643).  Returns the generated text."""
    tokens = tokenizer.encode(prompt)
    current = 0
    for i, t in enumerate(tokens):
        current = forward(t, i)
    pos, text = len(tokens), []
    for _ in range(max_tokens):
        if current in (IM_END, 151643):
            break
        word = tokenizer.decode([current])
        if word and write is not None:
            write(word)
        text.append(word)
        current = forward(current, pos)
        pos += 1
    return "".join(text)
