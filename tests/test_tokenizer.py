"""The host tokenizer (hotseat_b200/tok.py) against hs-engine tok.rs: the
reference's own unit-test vectors for the pre-tokenizer and the byte map
(tok.rs:351-416), BPE merges by rank, control tokens matched literally,
byte-exact decode round trips, and the vocabulary read from a GGUF."""
import numpy as np

from hotseat_b200 import tok
from tests.golden.synth import write_synthetic_gguf


def p(s):
    return tok.pretokenize(s)


def test_reference_pretokenizer_vectors():
    assert p("Hello world") == ["Hello", " world"]
    assert p("the quick brown fox") == ["the", " quick", " brown", " fox"]
    assert p("x=1234") == ["x", "=", "1", "2", "3", "4"]
    assert p("don't") == ["don", "'t"]
    assert p("They'RE here") == ["They", "'RE", " here"]
    assert p("I'll've") == ["I", "'ll", "'ve"]
    assert p("a   ") == ["a", "   "]
    assert p("a   b") == ["a", "  ", " b"]
    assert p("a  \n\nb") == ["a", "  \n\n", "b"]
    assert p("a\n  b") == ["a", "\n", " ", " b"]
    assert p("wow!!! ok") == ["wow", "!!!", " ok"]
    assert p("f(x) -> y") == ["f", "(x", ")", " ->", " y"]
    assert p("a.b") == ["a", ".b"]
    for s in ["", "a", "  ", "\n", "\r\n\r\n", "héllo wörld 42!", "  leading", "tab\there"]:
        assert "".join(p(s)) == s


def test_every_character_is_accounted_for_on_random_text():
    rng = np.random.default_rng(0)
    alphabet = list("abcXYZ019 '\t\n\r!?.,-()éßΩж中日😀") + [" ", " ", "́", "٣", "Ⅷ"]
    for _ in range(200):
        s = "".join(rng.choice(alphabet, size=int(rng.integers(0, 40))))
        assert "".join(p(s)) == s


def test_unicode_classes_follow_rust_char():
    # Alphabetic includes combining vowel signs (Other_Alphabetic) and letter
    # numbers; numeric is Nd/Nl/No; whitespace is White_Space
    assert tok.is_letter("ा") and tok.is_letter("Ⅷ") and tok.is_letter("é")
    assert tok.is_number("Ⅷ") and tok.is_number("½") and tok.is_number("٣")
    assert not tok.is_number("一")
    assert tok.is_space(" ") and tok.is_space(" ") and not tok.is_space("​")


def test_byte_map_is_a_bijection():
    b2u, u2b = tok.byte_to_unicode()
    assert len(u2b) == 256 and all(u2b[b2u[b]] == b for b in range(256))
    assert b2u[ord(" ")] == "Ġ" and b2u[ord("\n")] == "Ċ"


def _toy():
    b2u, _ = tok.byte_to_unicode()
    vocab = list(b2u)
    merges = ["Ġ t", "h e", "Ġt he", "l l", "ll o", "Ġ w"]
    for m in merges:
        a, b = m.split(" ")
        vocab.append(a + b)
    vocab += ["<|im_start|>", "<|im_end|>", "<|unused|>"]
    types = [1] * (len(vocab) - 3) + [3, 3, 1]
    return tok.Tokenizer(vocab, merges, types, eos=len(vocab) - 2)


def test_bpe_merges_by_rank_and_specials_match_literally():
    t = _toy()
    ids = t.encode("hello the world")
    pieces = [t.vocab[i] for i in ids]
    assert pieces == ["he", "llo", "Ġthe", "Ġw", "o", "r", "l", "d"]
    ids = t.encode("<|im_start|>the<|im_end|><|unused|>")
    assert ids[0] == t.id_of("<|im_start|>") and t.id_of("<|im_end|>") in ids
    assert t.id_of("<|unused|>") not in ids  # not a control token: byte-encoded
    assert t.decode(ids) == "<|im_start|>the<|im_end|><|unused|>"


def test_decode_round_trips_any_text():
    t = _toy()
    rng = np.random.default_rng(1)
    alphabet = list("hello world the \n\t!?éж中😀'sre") + ["<|im_end|>"]
    for _ in range(100):
        s = "".join(rng.choice(alphabet, size=int(rng.integers(0, 30))))
        assert t.decode(t.encode(s)) == s


def test_vocabulary_from_the_gguf(tmp_path):
    path = str(tmp_path / "t.gguf")
    write_synthetic_gguf(path, n_layers=1, d_model=128, n_heads=2, n_kv_heads=1, d_ff=256, vocab=300, seed=3, eos=299)
    t = tok.Tokenizer.from_gguf(path)
    assert t.vocab_size() == 300 and t.eos == 299 and t.bos is None
    assert t.id_of("<t17>") == 17 and t.token_text(17) == "<t17>"
