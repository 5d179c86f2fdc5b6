"""Hugging Face tokenizer.json loading (``Tokenizer.from_json``): a byte-level BPE vocabulary with the
Llama-3 split regex encodes and decodes exactly as the same vocabulary loaded from GGUF metadata;
tokenizer_config.json sets bos / eos / add_bos; a Unigram vocabulary is SentencePiece with scores."""
import json

import pytest

from hawking_b200._ext import native  # noqa: E402

LLAMA3_RE = ("(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}{1,3}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|"
             "\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+")
TEXTS = ["hello world", "The year 2024 had 366 days!", "  spaces\tand\ttabs\n\nnew lines", "ünïcödé ☃ 漢字",
         "<|begin_of_text|>Hi<|eot_id|>", ""]


def _bpe_files(tmp_path, with_config=True):
    from hawking_b200.formats.synth import synthetic_bpe_vocab, write_tokenizer_gguf
    toks, merges, bos, eos = synthetic_bpe_vocab(1024)
    tj = {"version": "1.0", "model": {"type": "BPE", "vocab": {t: i for i, t in enumerate(toks)},
                                      "merges": [m.split(" ", 1) for m in merges]},
          "pre_tokenizer": {"type": "Sequence", "pretokenizers": [
              {"type": "Split", "pattern": {"Regex": LLAMA3_RE}, "behavior": "Isolated", "invert": False},
              {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False}]},
          "added_tokens": [{"id": bos, "content": toks[bos], "special": True},
                           {"id": eos, "content": toks[eos], "special": True}]}
    p = tmp_path / "tokenizer.json"
    p.write_text(json.dumps(tj))
    c = tmp_path / "tokenizer_config.json"
    c.write_text(json.dumps({"bos_token": toks[bos], "eos_token": {"content": toks[eos]}, "add_bos_token": True}))
    g = write_tokenizer_gguf(str(tmp_path / "tok.gguf"), 1024)
    return str(p), str(c) if with_config else "", g


def test_bpe_tokenizer_json_matches_gguf(tmp_path):
    pj, pc, g = _bpe_files(tmp_path)
    a = native().Tokenizer.from_json(pj, pc)
    b = native().Tokenizer.from_gguf(native().GgufFile.open(g))
    assert a.vocab_size == b.vocab_size
    assert (a.bos, a.eos) == (b.bos, b.eos)
    for t in TEXTS:
        ids = a.encode(t, True)
        assert ids == b.encode(t, True), t
        assert a.decode(ids) == b.decode(ids)
    assert a.is_eog(a.eos)


def test_unigram_tokenizer_json(tmp_path):
    vocab = [["<unk>", 0.0], ["<s>", 0.0], ["</s>", 0.0]] + [[f"<0x{i:02X}>", 0.0] for i in range(256)]
    pieces = ["▁", "▁h", "▁he", "▁hel", "▁hell", "▁hello", "e", "l", "o", "h", "w",
              "▁w", "▁wo", "▁wor", "▁worl", "▁world", "r", "d"]
    vocab += [[p, -float(i)] for i, p in enumerate(pieces)]
    tj = {"model": {"type": "Unigram", "unk_id": 0, "vocab": vocab}, "added_tokens": [
        {"id": 1, "content": "<s>", "special": True}, {"id": 2, "content": "</s>", "special": True}]}
    p = tmp_path / "tokenizer.json"
    p.write_text(json.dumps(tj))
    c = tmp_path / "tokenizer_config.json"
    c.write_text(json.dumps({"bos_token": "<s>", "eos_token": "</s>"}))
    t = native().Tokenizer.from_json(str(p), str(c))
    assert t.is_spm
    ids = t.encode("hello world", True)
    assert ids[0] == 1  # SentencePiece vocabularies add bos by default
    assert t.decode(ids) == "hello world"
    assert t.encode("hello world", False) == [t.find("▁hello"), t.find("▁world")]


def test_tokenizer_json_rejects_unknown_model(tmp_path):
    p = tmp_path / "tokenizer.json"
    p.write_text(json.dumps({"model": {"type": "WordPiece", "vocab": {"a": 0}}}))
    with pytest.raises(Exception):
        native().Tokenizer.from_json(str(p))
