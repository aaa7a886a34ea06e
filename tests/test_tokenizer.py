import numpy as np

from krunch_b200.tokenizer import ByteTokenizer, load_tokenizer, tokenizer_for_id


def test_byte_tokenizer_lossless():
    t = ByteTokenizer()
    raw = bytes(range(256)) * 3 + "héllo ✓".encode() + b"\xff\xfe"
    ids = t.encode(raw)
    assert ids.dtype == np.int32 and len(ids) == len(raw)
    assert t.decode(ids) == raw
    assert tokenizer_for_id(2).name == "byte"


def test_default_without_tokenizer_file(monkeypatch, tmp_path):
    monkeypatch.setenv("KRUNCH_MODEL_DIR", str(tmp_path))
    monkeypatch.delenv("KRUNCH_TOKENIZER", raising=False)
    assert load_tokenizer().tokenizer_id == 2
