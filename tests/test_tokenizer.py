"""GGUF-vocabulary tokenizer: byte-level BPE and SentencePiece modes, special tokens, streaming.

Parity: crates/hawking-core/src/tokenizer.rs (from_gguf :156, encode :241, decode :266, is_eog :309,
SentencePiece bigram merge :441-548 and its tests :946-1020).
"""
import pytest

from hawking_b200.formats.gguf import GgufBuilder


def gpt2_byte_alphabet():
    """Printable bytes keep their code point, the other 68 map to U+0100.. in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


B2U = gpt2_byte_alphabet()
SPECIALS = ["<|begin_of_text|>", "<|eot_id|>", "<|start_header_id|>", "<|end_header_id|>"]
MERGES = ["Ġ t", "h e", "Ġt he", "t he", "l l", "Ġ w", "o r", "Ġw or", "l d", "Ġwor ld", "H e", "He ll", "Hell o"]


def bpe_spec(native):
    toks = [B2U[b] for b in range(256)]
    for m in MERGES:
        a, b = m.split(" ")
        toks.append(a + b)
    toks += SPECIALS
    sp = native.TokenizerSpec()
    sp.model = "gpt2"
    sp.pre = "llama-bpe"
    sp.tokens = toks
    sp.merges = MERGES
    sp.bos = toks.index("<|begin_of_text|>")
    sp.eos = toks.index("<|eot_id|>")
    return sp


def test_pretokenize_gpt2_and_llama3(native):
    assert native.pretokenize("Hello world's 123  x\n", "default") == ["Hello", " world", "'s", " 123", " ", " x", "\n"]
    assert native.pretokenize("Hello world's 1234567", "llama-bpe") == ["Hello", " world", "'s", " ", "123", "456", "7"]
    assert native.pretokenize("a,  b!!\n\nc", "llama-bpe") == ["a", ",", " ", " b", "!!\n\n", "c"]
    assert native.pretokenize("x 12345", "qwen2") == ["x", " ", "1", "2", "3", "4", "5"]
    assert native.pretokenize("I'LL go", "llama-bpe") == ["I", "'LL", " go"]


def test_bpe_merges_specials_roundtrip(native):
    sp = bpe_spec(native)
    tok = native.Tokenizer.from_spec(sp)
    assert tok.add_bos  # "llama-bpe" defaults to a BOS
    ids = tok.encode("Hello the world", add_special=False)
    assert [tok.token(i) for i in ids] == ["Hello", "Ġthe", "Ġworld"]
    ids = tok.encode("<|begin_of_text|>the<|eot_id|>", add_special=False)
    assert ids[0] == sp.bos and ids[-1] == sp.eos and [tok.token(i) for i in ids[1:-1]] == ["the"]
    assert tok.encode("hi")[0] == sp.bos
    assert tok.is_eog(sp.eos) and tok.is_special(sp.bos) and not tok.is_eog(ids[1])
    for text in ["plain ascii text", "naïve café ünïcödé", "中文字符 and emoji 🎉🚀", "tabs\tand\nnewlines\r\n  x",
                 "<|eot_id|> inside text"]:
        ids = tok.encode(text, add_special=False)
        assert tok.decode(ids, skip_special=False) == text
    assert tok.decode(tok.encode("a<|eot_id|>b", add_special=False), skip_special=True) == "ab"


def test_stream_decoder_holds_partial_utf8(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    ids = tok.encode("é🎉", add_special=False)  # byte tokens: 2 + 4 bytes
    assert len(ids) == 6
    sd = native.StreamDecoder(tok)
    outs = [sd.push(i) for i in ids]
    assert outs[0] == b"" and outs[1] == "é".encode()
    assert outs[2:5] == [b"", b"", b""] and outs[5] == "🎉".encode()
    assert sd.flush() == b""


def spm_spec(native):
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    words = ["▁", "a", "b", "c", "▁a", "ab", "▁ab", "▁b", "▁c", "bc", "▁abc"]
    scores = [0.0] * len(pieces) + [-5.0, -3.0, -3.0, -3.0, -2.0, -2.5, -1.0, -2.0, -2.0, -2.2, -0.5]
    sp = native.TokenizerSpec()
    sp.model = "llama"
    sp.tokens = pieces + words
    sp.scores = scores
    sp.token_types = [2, 3, 3] + [6] * 256 + [1] * len(words)
    sp.bos, sp.eos, sp.unk = 1, 2, 0
    return sp


def test_sentencepiece_scores_and_byte_fallback(native):
    tok = native.Tokenizer.from_spec(spm_spec(native))
    assert tok.is_spm and tok.add_bos
    ids = tok.encode("abc ab", add_special=False)
    assert [tok.token(i) for i in ids] == ["▁abc", "▁ab"]
    ids = tok.encode("ax", add_special=False)  # 'x' is not in the vocabulary: byte fallback
    assert [tok.token(i) for i in ids] == ["▁a", "<0x78>"]
    assert tok.decode(ids) == "ax"
    assert tok.encode("ab")[0] == 1
    assert tok.is_eog(2)


def test_tokenizer_from_gguf(native, tmp_path):
    sp = bpe_spec(native)
    b = GgufBuilder("llama")
    b.set("tokenizer.ggml.model", "gpt2")
    b.set("tokenizer.ggml.pre", "llama-bpe")
    b.set("tokenizer.ggml.tokens", list(sp.tokens))
    b.set("tokenizer.ggml.merges", list(sp.merges))
    b.set("tokenizer.ggml.bos_token_id", sp.bos, 4)
    b.set("tokenizer.ggml.eos_token_id", sp.eos, 4)
    b.set("tokenizer.ggml.add_bos_token", False)
    import numpy as np
    b.add("token_embd.weight", np.zeros((4, 32), np.float32))
    path = b.write(tmp_path / "tok.gguf")
    f = native.GgufFile.open(str(path))
    tok = native.Tokenizer.from_gguf(f)
    assert not tok.add_bos
    assert [tok.token(i) for i in tok.encode("Hello the world")] == ["Hello", "Ġthe", "Ġworld"]


def test_tokenizer_only_gguf_roundtrip(tmp_path, native):
    """The tensor-less synthetic tokenizer file (served with random-weight presets)."""
    from hawking_b200.formats.synth import write_tokenizer_gguf
    p = write_tokenizer_gguf(str(tmp_path / "tok.gguf"), 4096)
    tok = native.Tokenizer.from_gguf(native.GgufFile.open(p))
    ids = tok.encode("hello world, 123")
    assert ids and max(ids) < 4096
    assert tok.decode(ids) == "hello world, 123"
