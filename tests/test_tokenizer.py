"""Package tokenizer (jfb_tokenizer_*, include/jetsonfabric/tokenizer.hpp).

The reference tokenizes with llama.cpp's vocabulary code
(runtime/adapters/llama_cpp_tokenizer.cpp), which is not present here. The
byte-level BPE it runs for Qwen2 vocabularies is a published algorithm (GPT-2
byte-to-unicode mapping, the Qwen2 pre-tokenizer pattern, rank-ordered
merges, special tokens cut out first), so these tests pin this implementation
against an independent one of the same algorithm: the Hugging Face
`tokenizers` library, configured as Qwen2's tokenizer.json is (Split on the
pattern, ByteLevel without its own regex, BPE). A small vocabulary is trained
here on seeded multilingual text; its tokens, merges and token types are
written into a package's metadata.gguf under the GGUF tokenizer keys, and both
implementations must produce the same ids for seeded random texts and edge
cases. Parity with llama.cpp itself is therefore not pinned.
"""
from __future__ import annotations

import json
import random
import struct

import pytest

from jetsonfabric_b200 import jfm

tokenizers = pytest.importorskip("tokenizers")

QWEN2_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
                 r"|\s*[\r\n]+|\s+(?!\S)|\s+")
# the "llama-bpe" pre-tokenizer: the same pattern with digits in runs of up to three
LLAMA_BPE_PATTERN = QWEN2_PATTERN.replace(r"|\p{N}|", r"|\p{N}{1,3}|")
SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]

WORDS = ["the", "The", "quick", "brown", "fox", "jumps", "over", "lazy", "dog", "don't", "I'LL", "we've", "You'Re",
         "it's", "'s", "'d", "hello", "world", "tokenizer", "B200", "GPU", "naïve", "café", "Straße", "über",
         "Привет", "мир", "Ελληνικά", "中文", "分词器", "日本語", "かな", "한국어", "العربية", "😀", "🚀", "１２３",
         "²", "Ⅻ", "x²", "3.14159", "1,000,000", "2026", "e=mc²", "a_b", "#hash", "@user", "http://x.y/z?a=1",
         "(parens)", "[brackets]", "{braces}", "...", "!!!", "?!", "--", "—", "“quoted”", " nbsp"]
SPACES = [" ", " ", " ", "  ", "   ", "\t", "\n", "\n\n", "\r\n", " \n", "\n ", "　", " "]


def random_text(rng: random.Random, n: int) -> str:
    parts = []
    for _ in range(n):
        parts.append(rng.choice(WORDS))
        parts.append(rng.choice(SPACES))
        if rng.random() < 0.05:
            parts.append(rng.choice(SPECIALS))
    return "".join(parts)


def gguf_metadata(kv: list) -> bytes:
    """A GGUF v3 prefix with no tensors: kv = [(key, kind, value)], kind in
    'str', 'u32', 'bool', 'str[]', 'i32[]'."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 0, len(kv)))

    def string(s: str):
        b = s.encode()
        out.extend(struct.pack("<Q", len(b)) + b)

    for key, kind, value in kv:
        string(key)
        if kind == "str":
            out.extend(struct.pack("<I", 8))
            string(value)
        elif kind == "u32":
            out.extend(struct.pack("<II", 4, value))
        elif kind == "bool":
            out.extend(struct.pack("<IB", 7, int(value)))
        elif kind == "str[]":
            out.extend(struct.pack("<IIQ", 9, 8, len(value)))
            for s in value:
                string(s)
        elif kind == "i32[]":
            out.extend(struct.pack("<IIQ", 9, 5, len(value)) + struct.pack(f"<{len(value)}i", *value))
    return bytes(out + b"\0" * (-len(out) % 32))


def train(pattern: str):
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers

    rng = random.Random(7)
    corpus = [random_text(rng, 40) for _ in range(400)]
    hf = Tokenizer(models.BPE())
    hf.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(pattern), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False)])
    hf.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1200, special_tokens=SPECIALS, show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    hf.train_from_iterator(corpus, trainer)
    model = json.loads(hf.to_str())["model"]
    vocab = sorted(model["vocab"].items(), key=lambda kv: kv[1])
    assert [i for _, i in vocab] == list(range(len(vocab)))
    tokens = [t for t, _ in vocab]
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    return hf, tokens, merges


@pytest.fixture(scope="module")
def trained():
    return train(QWEN2_PATTERN)


def write_package(tmp_path, tokens, merges, extra=(), pre="qwen2", model="gpt2"):
    types = [3 if t in SPECIALS else 1 for t in tokens]
    kv = [("general.architecture", "str", "qwen2"), ("tokenizer.ggml.model", "str", model),
          ("tokenizer.ggml.pre", "str", pre), ("tokenizer.ggml.tokens", "str[]", tokens),
          ("tokenizer.ggml.token_type", "i32[]", types), ("tokenizer.ggml.merges", "str[]", merges),
          ("tokenizer.ggml.bos_token_id", "u32", tokens.index("<|endoftext|>")),
          ("tokenizer.ggml.eos_token_id", "u32", tokens.index("<|im_end|>")),
          ("tokenizer.ggml.add_bos_token", "bool", False)] + list(extra)
    d = tmp_path / "pkg"
    d.mkdir(parents=True, exist_ok=True)
    (d / "metadata.gguf").write_bytes(gguf_metadata(kv))
    return d


EDGE_CASES = [
    "Hello world", " Hello", "  Hello", "Hello  ", "Hello\n", "\n\nHello", "a\r\nb", "a \n b", " \n\n x",
    "don't DON'T Don'T", "'s'S'll", "x'ss", "123456", "１２３４", "x²³", "3.14", "   ", "\t\t", "!!!???",
    " ...", "a...b", "中文分词器测试", "naïve café", "😀😀 🚀", "<|im_start|>user\nhi<|im_end|>",
    "<|im_end|><|endoftext|>", "x<|im_start|>y", "<|im_start", "e=mc²", "http://x.y/z?a=1", "  a",
    "a　b", "  ", "the_quick", "Привет, мир!", "Ⅻ and ⅻ",
]


def test_matches_hf_byte_level_bpe(trained, tmp_path):
    hf, tokens, merges = trained
    tok = jfm.Tokenizer(write_package(tmp_path, tokens, merges))
    rng = random.Random(11)
    texts = EDGE_CASES + [random_text(rng, rng.randint(1, 60)) for _ in range(300)]
    for text in texts:
        assert tok.tokenize(text) == hf.encode(text).ids, repr(text)


def test_llama_bpe_pre_tokenizer_matches_hf(tmp_path):
    """The "llama-bpe" pre-tokenizer (digit runs of up to three) against the
    same published pattern in Hugging Face `tokenizers`, on a vocabulary
    trained with it."""
    hf, tokens, merges = train(LLAMA_BPE_PATTERN)
    assert LLAMA_BPE_PATTERN != QWEN2_PATTERN
    tok = jfm.Tokenizer(write_package(tmp_path, tokens, merges, pre="llama-bpe"))
    rng = random.Random(13)
    digits = ["1234567", "x12345y", "2026-12-02", "3.14159265", "1,000,000", "１２３４５", "42 42 4242", "007"]
    texts = EDGE_CASES + digits + [random_text(rng, rng.randint(1, 60)) for _ in range(200)]
    for text in texts:
        assert tok.tokenize(text) == hf.encode(text).ids, repr(text)
    # the two pre-tokenizers split digit runs differently
    qwen2 = jfm.Tokenizer(write_package(tmp_path / "q", tokens, merges, pre="qwen2"))
    assert len(qwen2.tokenize("1234567")) >= len(tok.tokenize("1234567"))


def test_pieces_round_trip_the_text(trained, tmp_path):
    hf, tokens, merges = trained
    tok = jfm.Tokenizer(write_package(tmp_path, tokens, merges))
    rng = random.Random(12)
    for text in EDGE_CASES + [random_text(rng, 30) for _ in range(50)]:
        ids = tok.tokenize(text)
        assert b"".join(tok.token_piece(i) for i in ids) == text.encode(), repr(text)


def test_end_tokens_and_bos(trained, tmp_path):
    _, tokens, merges = trained
    tok = jfm.Tokenizer(write_package(tmp_path, tokens, merges))
    assert tok.is_end_token(tokens.index("<|im_end|>"))
    assert tok.is_end_token(tokens.index("<|endoftext|>"))
    assert tok.is_end_token(-1)
    assert not tok.is_end_token(tokens.index("<|im_start|>"))
    assert not tok.is_end_token(tok.tokenize("hello")[0])
    assert tok.token_piece(tokens.index("<|im_start|>")) == b"<|im_start|>"
    assert tok.tokenize("hi")[0] != tokens.index("<|endoftext|>")
    # add_bos_token = true prepends the BOS id
    kv_bos = write_package(tmp_path / "bos", tokens, merges)
    meta = (kv_bos / "metadata.gguf").read_bytes()
    (kv_bos / "metadata.gguf").write_bytes(meta.replace(b"tokenizer.ggml.add_bos_token\x07\x00\x00\x00\x00",
                                                        b"tokenizer.ggml.add_bos_token\x07\x00\x00\x00\x01"))
    assert jfm.Tokenizer(kv_bos).tokenize("hi")[0] == tokens.index("<|endoftext|>")


def test_truncated_metadata_is_rejected(trained, tmp_path):
    """Prefixes of a tokenizer's metadata.gguf (every 5th length and the last
    64) raise JfmError; none reads past the end."""
    _, tokens, merges = trained
    d = write_package(tmp_path, tokens, merges)
    meta = (d / "metadata.gguf").read_bytes()
    cut = tmp_path / "cut"
    cut.mkdir()
    lengths = sorted(set(range(0, len(meta), 5)) | set(range(max(0, len(meta) - 64), len(meta))))
    for n in lengths:
        (cut / "metadata.gguf").write_bytes(meta[:n])
        try:
            jfm.Tokenizer(cut)
        except jfm.JfmError:
            continue
        # only a prefix that ends in the zero padding after the last value can parse
        assert meta[n:].strip(b"\0") == b"", n


CPP_CONSUMER = r"""
#include "jetsonfabric/tokenizer.hpp"

#include <cstdio>
#include <stdexcept>
#include <string>

int main(int argc, char ** argv) {
    if (argc != 3) return 2;
    const auto tok = jetsonfabric::native::open_package_tokenizer(argv[1]);
    const std::string text = argv[2];
    std::string joined;
    for (const std::int32_t id : tok->tokenize(text)) {
        std::printf("%d ", id);
        joined += tok->token_piece(id);
    }
    std::printf("\n%s\n%d\n", joined == text ? "round-trip" : "mismatch", tok->is_end_token(-1) ? 1 : 0);
    try {
        (void) tok->tokenize("");
        std::printf("accepted\n");
    } catch (const std::invalid_argument &) {
        std::printf("invalid_argument\n");
    }
    try {
        (void) jetsonfabric::native::open_package_tokenizer(std::string(argv[1]) + "/missing");
        std::printf("accepted\n");
    } catch (const std::invalid_argument &) {
        std::printf("invalid_argument\n");
    }
    return 0;
}
"""


def test_cpp_interface_matches_the_c_abi(trained, tmp_path):
    """A C++ caller of the reference's Tokenizer interface
    (include/jetsonfabric/tokenizer.hpp) linked against libjfm.so gets the
    ids of the C ABI, the documented exceptions, and round-tripping pieces."""
    import shutil
    import subprocess
    from pathlib import Path

    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    jfm.lib()  # builds libjfm.so if needed
    repo = Path(__file__).resolve().parent.parent
    lib_dir = repo / "jetsonfabric_b200" / "lib"
    src = tmp_path / "consumer.cpp"
    src.write_text(CPP_CONSUMER)
    exe = tmp_path / "consumer"
    subprocess.run(["g++", "-std=c++20", "-O1", f"-I{repo / 'include'}", str(src), "-o", str(exe), f"-L{lib_dir}",
                    "-ljfm", f"-Wl,-rpath,{lib_dir}"], check=True)
    _, tokens, merges = trained
    d = write_package(tmp_path, tokens, merges)
    text = "Hello world, naïve café <|im_start|>user 12345"
    out = subprocess.run([str(exe), str(d), text], check=True, capture_output=True, text=True).stdout.split("\n")
    assert [int(x) for x in out[0].split()] == jfm.Tokenizer(d).tokenize(text)
    assert out[1:5] == ["round-trip", "1", "invalid_argument", "invalid_argument"]


def test_rejections(trained, tmp_path):
    _, tokens, merges = trained
    with pytest.raises(jfm.JfmError, match="metadata.gguf"):
        jfm.Tokenizer(tmp_path)
    with pytest.raises(jfm.JfmError, match="not supported"):
        jfm.Tokenizer(write_package(tmp_path / "spm", tokens, merges, model="llama"))
    with pytest.raises(jfm.JfmError, match="not supported"):
        jfm.Tokenizer(write_package(tmp_path / "pre", tokens, merges, pre="falcon"))
    tok = jfm.Tokenizer(write_package(tmp_path / "ok", tokens, merges))
    with pytest.raises(jfm.JfmError, match="no tokens"):
        tok.tokenize("")
    with pytest.raises(jfm.JfmError, match="outside the vocabulary"):
        tok.token_piece(len(tokens))
