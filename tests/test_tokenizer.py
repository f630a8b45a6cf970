"""Host tokenizer parity: vrt_tokenize / vrt_token_piece (the C++
Gemma3Tokenizer) against the reference's own Gemma3Model::tokenize and
piece decoding (oracle/_ref), on the synthetic vocabularies."""

import pytest

import oracle as O
import synth_gguf as sg
import vrt

TEXTS = ["Hello", "Hello world", "  Hello   world\tand\nthe token ", "Gemma on B200 is a token",
         "café ☃ <t300> \x01", "", "abc" * 40, "<0x41>", "▁the"]


@pytest.fixture(scope="module", params=["tiny", "270m"])
def vocab_model(request, model_dir):
    shape = sg.SHAPES[request.param]
    if request.param == "270m":
        shape = shape.with_(block_count=1, name="270m-tok")  # full vocabulary, one layer
    return sg.cached_model(shape, 5, model_dir)


@pytest.mark.skipif(not O.reference_available(), reason="oracle/_ref not built")
def test_tokenize_matches_reference(vocab_model):
    tok = vrt.Tokenizer(vocab_model)
    ref = O.Reference(vocab_model)
    for t in TEXTS:
        for bos in (True, False):
            assert tok.tokenize(t, bos) == ref.tokenize(t, bos), t


def test_pieces(vocab_model):
    tok = vrt.Tokenizer(vocab_model)
    toks, _, _ = sg.vocab_pieces(768)
    assert tok.piece(2) == b"<bos>" and tok.piece(2, decoded=True) == b""
    assert tok.piece(4 + 0x41, decoded=True) == b"A"
    idx = toks.index("▁Hello")
    assert tok.piece(idx, decoded=True) == b" Hello"
    assert tok.tokenize("Hello")[0] == 2


def test_tokenizer_errors(tmp_path):
    with pytest.raises(vrt.VrtError):
        vrt.Tokenizer(str(tmp_path / "missing.gguf"))
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF\x09\x00\x00\x00" + b"\x00" * 16)
    with pytest.raises(vrt.VrtError, match="version"):
        vrt.Tokenizer(str(bad))
