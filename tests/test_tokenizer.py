"""Qwen tokenizer (QwenTokenizer.swift, main.swift:11-13) against Hugging Face
`tokenizers` (the library swift-transformers ports) on byte-level BPE
tokenizers trained here from a synthetic corpus with the Qwen2 pre-tokenizer
(split regex, NFC, byte level) and Qwen's special tokens.  No tokenizer.json of
the real model exists in this environment; the checks are that this module's
encode and decode equal the library's on the same file, that the streaming
decoder holds incomplete UTF-8 sequences back, and that ChatML prompts encode
as the reference splits them.
"""
import json
import random

import pytest

tokenizers = pytest.importorskip("tokenizers")

from qweninferenceengine_b200.tokenizer import (  # noqa: E402
    IM_END, IM_START, BPETokenizer, QwenTokenizer, byte_level_table, format_prompt)

QWEN_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
              r"|\s*[\r\n]+|\s+(?!\S)|\s+")
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def corpus(seed, n=400):
    rnd = random.Random(seed)
    words = ["hello", "world", "the", "tokenizer", "Qwen", "B200", "don't", "we'll", "ÜBER", "café",
             "naïve", "数据", "模型", "推理", "😀", "ünïcödé", "x86_64", "1234567", "foo.bar()", "\t",
             "    ", "\n\n", "can't", "I'M", "résumé", "Ελληνικά", "русский", "#include", "<tag>"]
    out = []
    for _ in range(n):
        out.append(" ".join(rnd.choice(words) for _ in range(rnd.randint(1, 12))))
    return out


def train(tmp_path, seed, vocab_size):
    from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers

    tok = Tokenizer(models.BPE())
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=SPECIAL,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  show_progress=False)
    tok.train_from_iterator(corpus(seed), trainer=trainer)
    d = tmp_path / f"tok{seed}_{vocab_size}"
    d.mkdir()
    tok.save(str(d / "tokenizer.json"))
    return tok, d


TEXTS = ["hello world", "Hello World!!", "don't stop, we'll go; I'M here", "café naïve résumé",
         "数据模型推理", "😀😀 x86_64\tfoo.bar()", "   leading and trailing   ", "a\n\nb\r\n  c",
         "1234567890 12 3", "ünïcödé Ελληνικά русский", "#include <tag>", "", " ", "\n",
         "unseen words zebra quux", "é composed", "It's 2026: the B200 runs Qwen."]


@pytest.mark.parametrize("seed,vocab", [(1, 300), (2, 700), (3, 2000)])
def test_encode_decode_match_the_library(tmp_path, seed, vocab):
    ref, d = train(tmp_path, seed, vocab)
    mine = BPETokenizer(str(d / "tokenizer.json"))
    rnd = random.Random(seed)
    texts = TEXTS + corpus(seed + 100, 60)
    alphabet = "ab cdé数😀\n\t'sZ9.!"
    texts += ["".join(rnd.choice(alphabet) for _ in range(rnd.randint(1, 30))) for _ in range(60)]
    for t in texts:
        assert mine.encode(t) == ref.encode(t).ids, repr(t)
    n = ref.get_vocab_size()
    for _ in range(200):
        ids = [rnd.randrange(n) for _ in range(rnd.randint(1, 12))]
        assert mine.decode(ids) == ref.decode(ids, skip_special_tokens=False), ids


def test_byte_level_table_is_the_library_alphabet():
    from tokenizers import pre_tokenizers

    table = byte_level_table()
    assert sorted(table.values()) == sorted(pre_tokenizers.ByteLevel.alphabet())
    assert all(table[b] == chr(b) for b in range(ord("!"), ord("~") + 1))


def test_streaming_decode_holds_incomplete_utf8(tmp_path):
    ref, d = train(tmp_path, 4, 300)
    qt = QwenTokenizer(str(d))
    text = "数据 😀 café and 模型"
    ids = qt.tokenizer.encode(text)
    assert ids == ref.encode(text).ids
    pieces = [qt.decode([i]) for i in ids]
    assert "".join(pieces) == text
    assert "" in pieces                     # some token ended inside a multi-byte character
    assert all("�" not in p for p in pieces)


def test_chatml_encode_splits_the_tags(tmp_path):
    ref, d = train(tmp_path, 5, 500)
    qt = QwenTokenizer(str(d))
    prompt = format_prompt("What is a B200?")
    ids = qt.encode(prompt)
    want = []
    for i, part in enumerate(prompt.split("<|im_start|>")):
        if i:
            want.append(IM_START)
        for j, sub in enumerate(part.split("<|im_end|>")):
            if j:
                want.append(IM_END)
            if sub:
                want.extend(ref.encode(sub).ids)
    assert ids == want
    assert ids[0] == IM_START and ids.count(IM_START) == 3 and ids.count(IM_END) == 2


def test_missing_tokenizer_file(tmp_path):
    with pytest.raises(FileNotFoundError, match="Tokenizer weights file not found"):
        QwenTokenizer(str(tmp_path))


def test_added_tokens_are_matched_in_raw_text(tmp_path):
    ref, d = train(tmp_path, 6, 400)
    mine = BPETokenizer(str(d / "tokenizer.json"))
    t = "text<|endoftext|>more<|im_end|>"
    assert mine.encode(t) == ref.encode(t).ids
    cfg = json.loads((d / "tokenizer.json").read_text())
    ids = {a["content"]: a["id"] for a in cfg["added_tokens"]}
    assert mine.encode("<|endoftext|>") == [ids["<|endoftext|>"]]


def test_stream_generate_follows_the_reference_loop(tmp_path):
    """Positions 0..n-1 for the prompt, then one per generated token; text is
    written as it completes; <|im_end|> stops (its text is not written)."""
    from qweninferenceengine_b200.tokenizer import stream_generate

    ref, d = train(tmp_path, 7, 400)
    qt = QwenTokenizer(str(d))
    reply = ref.encode("数据 ok 😀").ids + [IM_END, 5, 6]
    calls = []

    def forward(tok, pos):
        calls.append((tok, pos))
        k = len(calls) - len(prompt_ids)       # 0 for the last prompt position
        return reply[k] if k >= 0 else 0

    prompt = format_prompt("hi")
    prompt_ids = qt.encode(prompt)
    qt2 = QwenTokenizer(str(d))
    written = []
    text = stream_generate(forward, qt2, prompt, max_tokens=64, write=written.append)
    assert text == "数据 ok 😀" and "".join(written) == text
    n = len(prompt_ids)
    assert [p for _, p in calls] == list(range(n + len(reply) - 3))
    assert [t for t, _ in calls[:n]] == prompt_ids
    assert [t for t, _ in calls[n:]] == reply[:len(reply) - 3]
    # max_tokens bounds the generated tokens
    calls.clear()
    assert stream_generate(forward, QwenTokenizer(str(d)), prompt, max_tokens=1, write=None) != text
